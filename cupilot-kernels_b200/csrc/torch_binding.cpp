// torch_binding.cpp — Torch C++ extension over the b2g C ABI.
//
// The reference ships one `torch::Tensor f(torch::Tensor A, torch::Tensor B)`
// per operator (its "Part 3" host wrapper).  This module exports one such
// function per operator, named after the operator, with the same argument
// meaning, output shape and dtype; the Python package re-exports each under
// `forward` and under the reference's own Part-3 name.  Every function
// validates its inputs with TORCH_CHECK, allocates the output with
// torch::empty (every element is written by the kernel), launches on the
// current CUDA stream and never synchronises the host.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <atomic>

#include "../../include/b2g_gemm.h"

namespace {

// Precision mode: a process-wide default (set_precision) and a per-thread
// override (set_thread_precision, used by the Python `precision()` context
// manager), so a scoped mode in one thread never changes another thread's
// calls.
std::atomic<int> g_precision{B2G_PREC_TF32};
thread_local int t_precision = -1;   // -1: no override, use the default

int precision_now() { return t_precision >= 0 ? t_precision : g_precision.load(); }

void check_status(int rc, const char* what) {
  TORCH_CHECK(rc == B2G_OK, what, ": ", b2g_status_string(rc), " (status ", rc, ")");
}

void check_input(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.scalar_type() == at::kFloat, name, " must be float32");
}

// A 2-D view as a GEMM operand: row-major with a pitch, or the transpose of
// one (column-major view), without copying.  Anything else is made
// contiguous first.
struct Operand {
  at::Tensor keep;
  const float* ptr;
  int64_t ld;
  int trans;   // 1: stored transposed relative to the logical matrix
};

Operand as_operand(const at::Tensor& t) {
  Operand o;
  const int64_t r = t.size(0), c = t.size(1);
  if (t.stride(1) == 1 && t.stride(0) >= std::max<int64_t>(c, 1)) {
    o.keep = t;
    o.ld = t.stride(0);
    o.trans = 0;
  } else if (t.stride(0) == 1 && t.stride(1) >= std::max<int64_t>(r, 1)) {
    o.keep = t;
    o.ld = t.stride(1);
    o.trans = 1;
  } else {
    o.keep = t.contiguous();
    o.ld = std::max<int64_t>(c, 1);
    o.trans = 0;
  }
  o.ptr = o.keep.data_ptr<float>();
  return o;
}

void run_gemm(b2g_gemm_desc& d, const at::Tensor& like) {
  const int64_t ws = b2g_gemm_workspace_bytes(&d);
  TORCH_CHECK(ws >= 0, "b2g: invalid GEMM descriptor");
  at::Tensor wst;
  if (ws > 0) {
    wst = at::empty({ws}, like.options().dtype(at::kByte));
    d.workspace = wst.data_ptr();
    d.workspace_bytes = ws;
  }
  auto stream = at::cuda::getCurrentCUDAStream(like.device().index());
  check_status(b2g_gemm(&d, stream.stream()), "b2g_gemm");
}

// C = A . B for logical 2-D matrices A (M x K) and B (K x N), either of
// which may be a transposed view; op selects the triangular variants.
at::Tensor matmul_2d(const at::Tensor& A, const at::Tensor& B, int op) {
  check_input(A, "A");
  check_input(B, "B");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2, "A and B must be 2-D");
  TORCH_CHECK(A.device() == B.device(), "A and B must be on the same device");
  TORCH_CHECK(A.size(1) == B.size(0), "inner dimensions differ: A is ", A.sizes(), ", B is ",
              B.sizes());
  const c10::cuda::CUDAGuard guard(A.device());
  const int64_t M = A.size(0), K = A.size(1), N = B.size(1);
  if (op != B2G_OP_GEMM)
    TORCH_CHECK(M == K && K == N, "triangular matmul needs square matrices of one size");
  at::Tensor C = at::empty({M, N}, A.options());
  if (M == 0 || N == 0) return C;
  if (K == 0) return C.zero_();
  Operand a = as_operand(A), b = as_operand(B);
  b2g_gemm_desc d{};
  d.op = op;
  d.precision = precision_now();
  d.m = M;
  d.n = N;
  d.k = K;
  d.batch = 1;
  d.a = a.ptr;
  d.lda = a.ld;
  d.trans_a = a.trans;
  d.b = b.ptr;
  d.ldb = b.ld;
  d.trans_b = b.trans;
  d.c = C.data_ptr<float>();
  d.ldc = N;
  run_gemm(d, A);
  return C;
}

// ---------------------------------------------------------------- operators
// kernels/1_Square_matrix_multiplication_best_kernel.cu:189 (matmul_cuda)
at::Tensor square_matmul(at::Tensor A, at::Tensor B) {
  TORCH_CHECK(A.dim() == 2 && A.size(0) == A.size(1), "A must be square");
  return matmul_2d(A, B, B2G_OP_GEMM);
}
// kernels/2_Standard_matrix_multiplication_best_kernel.cu:117 (matmul_cuda)
at::Tensor standard_matmul(at::Tensor A, at::Tensor B) { return matmul_2d(A, B, B2G_OP_GEMM); }
// kernels/6_Matmul_with_large_K_dimension_best_kernel.cu:128 (matmul_cuda)
at::Tensor large_k_matmul(at::Tensor A, at::Tensor B) { return matmul_2d(A, B, B2G_OP_GEMM); }
// kernels/7_Matmul_with_small_K_dimension_best_kernel.cu:80 (gemm_cuda)
at::Tensor small_k_matmul(at::Tensor A, at::Tensor B) { return matmul_2d(A, B, B2G_OP_GEMM); }
// kernels/8_Matmul_with_irregular_shapes_best_kernel.cu:155 (matmul_cuda)
at::Tensor irregular_matmul(at::Tensor A, at::Tensor B) { return matmul_2d(A, B, B2G_OP_GEMM); }
// kernels/9_Tall_skinny_matrix_multiplication_best_kernel.cu:145 (tall_skinny_matmul_cuda)
at::Tensor tall_skinny_matmul(at::Tensor A, at::Tensor B) { return matmul_2d(A, B, B2G_OP_GEMM); }
// kernels/16_Matmul_with_transposed_A_best_kernel.cu:124 — C = A^T B, A stored (K, M)
at::Tensor matmul_transposed_a(at::Tensor A, at::Tensor B) {
  TORCH_CHECK(A.dim() == 2, "A must be 2-D");
  return matmul_2d(A.t(), B, B2G_OP_GEMM);
}
// kernels/17_Matmul_with_transposed_B_best_kernel.cu:267 — C = A B^T, B stored (N, K)
at::Tensor matmul_transposed_b(at::Tensor A, at::Tensor B) {
  TORCH_CHECK(B.dim() == 2, "B must be 2-D");
  return matmul_2d(A, B.t(), B2G_OP_GEMM);
}
// kernels/18_Matmul_with_transposed_both_best_kernel.cu:152 — C = A^T B^T
at::Tensor matmul_transposed_both(at::Tensor A, at::Tensor B) {
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2, "A and B must be 2-D");
  return matmul_2d(A.t(), B.t(), B2G_OP_GEMM);
}
// kernels/13_Matmul_for_symmetric_matrices_best_kernel.cu:134 — B == B^T, so
// B is read K-major (as B^T) and both operands feed the MMA K-major.
at::Tensor symmetric_matmul(at::Tensor A, at::Tensor B) {
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && A.size(0) == A.size(1) && B.size(0) == B.size(1),
              "A and B must be square");
  return matmul_2d(A, B.t(), B2G_OP_GEMM);
}
// kernels/14_Matmul_for_upper_triangular_matrices_best_kernel.cu:135
at::Tensor upper_tri_matmul(at::Tensor A, at::Tensor B) {
  return matmul_2d(A, B, B2G_OP_TRI_UPPER);
}
// kernels/15_Matmul_for_lower_triangular_matrices_best_kernel.cu:155
at::Tensor lower_tri_matmul(at::Tensor A, at::Tensor B) {
  return matmul_2d(A, B, B2G_OP_TRI_LOWER);
}

// C[b] = A[b] B[b] into a caller-provided C (batch, M, N), row-major.
void batched_matmul_into(const at::Tensor& A, const at::Tensor& B, at::Tensor& C) {
  check_input(A, "A");
  check_input(B, "B");
  check_input(C, "C");
  TORCH_CHECK(A.dim() == 3 && B.dim() == 3, "A and B must be 3-D");
  TORCH_CHECK(A.size(0) == B.size(0) && A.size(2) == B.size(1), "bmm shape mismatch: ",
              A.sizes(), " x ", B.sizes());
  TORCH_CHECK(A.device() == B.device() && A.device() == C.device(),
              "A, B and C must be on the same device");
  const int64_t bs = A.size(0), M = A.size(1), K = A.size(2), N = B.size(2);
  TORCH_CHECK(C.dim() == 3 && C.size(0) == bs && C.size(1) == M && C.size(2) == N,
              "C must be (batch, M, N)");
  TORCH_CHECK(C.stride(2) == 1 && C.stride(1) >= std::max<int64_t>(N, 1) &&
                  (bs == 1 || C.stride(0) >= M * C.stride(1)),
              "C must be row-major per batch");
  const c10::cuda::CUDAGuard guard(A.device());
  if (bs == 0 || M == 0 || N == 0) return;
  if (K == 0) {
    C.zero_();
    return;
  }
  at::Tensor a = A.stride(2) == 1 ? A : A.contiguous();
  at::Tensor b = B.stride(2) == 1 ? B : B.contiguous();
  TORCH_CHECK(bs <= 65535, "batch too large");
  b2g_gemm_desc d{};
  d.op = B2G_OP_GEMM;
  d.precision = precision_now();
  d.m = M;
  d.n = N;
  d.k = K;
  d.batch = bs;
  d.a = a.data_ptr<float>();
  d.lda = std::max<int64_t>(a.stride(1), K);
  d.stride_a = bs > 1 ? a.stride(0) : 0;
  d.b = b.data_ptr<float>();
  d.ldb = std::max<int64_t>(b.stride(1), N);
  d.stride_b = bs > 1 ? b.stride(0) : 0;
  d.c = C.data_ptr<float>();
  d.ldc = C.stride(1);
  d.stride_c = bs > 1 ? C.stride(0) : 0;
  run_gemm(d, A);
}

// kernels/3_Batched_matrix_multiplication_best_kernel.cu:113 — C[b] = A[b] B[b]
at::Tensor batched_matmul(at::Tensor A, at::Tensor B) {
  check_input(A, "A");
  TORCH_CHECK(A.dim() == 3 && B.dim() == 3, "A and B must be 3-D");
  at::Tensor C = at::empty({A.size(0), A.size(1), B.size(2)}, A.options());
  batched_matmul_into(A, B, C);
  return C;
}

void batched_matmul_out(at::Tensor A, at::Tensor B, at::Tensor C) { batched_matmul_into(A, B, C); }

// kernels/10_3D_tensor_matrix_multiplication_best_kernel.cu:180 — out[n] = A[n] B,
// A (n, m, k), B (k, l): the batch folds into M (B is shared).
at::Tensor tensor3d_matmul(at::Tensor A, at::Tensor B) {
  check_input(A, "A");
  TORCH_CHECK(A.dim() == 3 && B.dim() == 2, "A must be 3-D and B 2-D");
  at::Tensor a = A.contiguous();
  at::Tensor C = matmul_2d(a.view({A.size(0) * A.size(1), A.size(2)}), B, B2G_OP_GEMM);
  return C.view({A.size(0), A.size(1), B.size(1)});
}

// kernels/11_4D_tensor_matrix_multiplication_best_kernel.cu:132 —
// einsum('bijl,lk->bijk'), returned as a (b, i, j, k) view like K11:165.
at::Tensor tensor4d_matmul(at::Tensor A, at::Tensor B) {
  check_input(A, "A");
  TORCH_CHECK(A.dim() == 4 && B.dim() == 2, "A must be 4-D and B 2-D");
  at::Tensor a = A.contiguous();
  at::Tensor C =
      matmul_2d(a.view({A.size(0) * A.size(1) * A.size(2), A.size(3)}), B, B2G_OP_GEMM);
  return C.view({A.size(0), A.size(1), A.size(2), B.size(1)});
}

// kernels/12_Matmul_with_diagonal_matrices_best_kernel.cu:43 — diag(A) . B
at::Tensor diag_matmul(at::Tensor A, at::Tensor B) {
  check_input(A, "A");
  check_input(B, "B");
  TORCH_CHECK(A.dim() == 1, "A must be 1-dimensional");
  TORCH_CHECK(B.dim() == 2, "B must be 2-dimensional");
  TORCH_CHECK(A.size(0) == B.size(0), "First dimension of B must match length of A");
  TORCH_CHECK(A.device() == B.device(), "A and B must be on the same device");
  const c10::cuda::CUDAGuard guard(A.device());
  at::Tensor d = A.contiguous();
  at::Tensor b = B.stride(1) == 1 ? B : B.contiguous();
  at::Tensor out = at::empty({B.size(0), B.size(1)}, B.options());
  auto stream = at::cuda::getCurrentCUDAStream(A.device().index());
  check_status(b2g_rowscale(d.data_ptr<float>(), b.data_ptr<float>(), out.data_ptr<float>(),
                            B.size(0), B.size(1), std::max<int64_t>(b.stride(0), B.size(1)),
                            B.size(1), stream.stream()),
               "b2g_rowscale");
  return out;
}

// kernels/4_Matrix_vector_multiplication_best_kernel.cu:84 — C (M, 1) = A (M, K) . B (K, 1)
at::Tensor gemv(at::Tensor A, at::Tensor B) {
  check_input(A, "A");
  check_input(B, "B");
  TORCH_CHECK(A.dim() == 2, "A must be 2D");
  TORCH_CHECK(B.dim() == 2, "B must be 2D");
  TORCH_CHECK(B.size(0) == A.size(1), "A and B shapes not matched");
  TORCH_CHECK(B.size(1) == 1, "B must be a column vector");
  TORCH_CHECK(A.device() == B.device(), "A and B must be on the same device");
  const c10::cuda::CUDAGuard guard(A.device());
  at::Tensor a = A.stride(1) == 1 ? A : A.contiguous();
  at::Tensor x = B.contiguous();
  at::Tensor C = at::empty({A.size(0), 1}, A.options());
  auto stream = at::cuda::getCurrentCUDAStream(A.device().index());
  check_status(b2g_gemv(a.data_ptr<float>(), std::max<int64_t>(a.stride(0), A.size(1)),
                        x.data_ptr<float>(), C.data_ptr<float>(), A.size(0), A.size(1),
                        stream.stream()),
               "b2g_gemv");
  return C;
}

// kernels/5_Matrix_scalar_multiplication_best_kernel.cu:47 — C = A * s
at::Tensor matrix_scalar_mult(at::Tensor A, double s) {
  check_input(A, "A");
  TORCH_CHECK(A.is_contiguous(), "A must be contiguous");
  const c10::cuda::CUDAGuard guard(A.device());
  at::Tensor C = at::empty_like(A);
  auto stream = at::cuda::getCurrentCUDAStream(A.device().index());
  check_status(b2g_scale(A.data_ptr<float>(), static_cast<float>(s), C.data_ptr<float>(),
                         A.numel(), stream.stream()),
               "b2g_scale");
  return C;
}

// kernels/87_conv_pointwise_2D_best_kernel.cu:451 (pointwise_conv_cuda) —
// out (N, Cout, H, W) = 1x1 convolution of input (N, Cin, H, W) with weight
// (Cout, Cin) or (Cout, Cin, 1, 1), plus an optional per-channel bias.
at::Tensor pointwise_conv(at::Tensor input, at::Tensor weight, c10::optional<at::Tensor> bias_opt);

// The reference also dispatches fp16 and bf16 (kernels/87_...:480-481): such
// inputs are widened to fp32, run through the same TF32 engine, and the
// output is returned in the input's dtype.
at::Tensor pointwise_conv_any(at::Tensor input, at::Tensor weight,
                              c10::optional<at::Tensor> bias_opt) {
  const auto dt = input.scalar_type();
  if (input.is_cuda() && (dt == at::kHalf || dt == at::kBFloat16)) {
    TORCH_CHECK(weight.scalar_type() == dt, "weight must have the input's dtype");
    c10::optional<at::Tensor> b32;
    if (bias_opt.has_value() && bias_opt->defined()) {
      TORCH_CHECK(bias_opt->scalar_type() == dt, "bias must have the input's dtype");
      b32 = bias_opt->to(at::kFloat);
    }
    return pointwise_conv(input.to(at::kFloat), weight.to(at::kFloat), b32).to(dt);
  }
  return pointwise_conv(input, weight, bias_opt);
}

at::Tensor pointwise_conv(at::Tensor input, at::Tensor weight, c10::optional<at::Tensor> bias_opt) {
  check_input(input, "input");
  check_input(weight, "weight");
  TORCH_CHECK(input.dim() == 4, "input must be (batch, in_channels, height, width)");
  TORCH_CHECK(weight.dim() == 2 || (weight.dim() == 4 && weight.size(2) == 1 && weight.size(3) == 1),
              "weight must be (out_channels, in_channels) or (out_channels, in_channels, 1, 1)");
  const int64_t bs = input.size(0), cin = input.size(1), h = input.size(2), w = input.size(3);
  const int64_t cout = weight.size(0);
  TORCH_CHECK(weight.size(1) == cin, "weight has ", weight.size(1), " input channels, input has ",
              cin);
  TORCH_CHECK(input.device() == weight.device(), "input and weight must be on the same device");
  at::Tensor bias;
  if (bias_opt.has_value() && bias_opt->defined()) {
    bias = *bias_opt;
    check_input(bias, "bias");
    TORCH_CHECK(bias.numel() == cout, "bias must have out_channels elements");
    TORCH_CHECK(bias.device() == input.device(), "bias must be on the input's device");
    bias = bias.contiguous();
  }
  const c10::cuda::CUDAGuard guard(input.device());
  at::Tensor out = at::empty({bs, cout, h, w}, input.options());
  if (out.numel() == 0) return out;
  TORCH_CHECK(bs <= 65535, "batch too large");
  at::Tensor x = input.contiguous();
  at::Tensor wt = weight.contiguous();
  const float* bp = bias.defined() ? bias.data_ptr<float>() : nullptr;
  const int prec = precision_now();
  const int64_t ws = b2g_pointwise_conv_workspace_bytes(x.data_ptr<float>(), wt.data_ptr<float>(),
                                                        out.data_ptr<float>(), bs, cin, cout,
                                                        h * w, prec);
  TORCH_CHECK(ws >= 0, "b2g: invalid pointwise convolution");
  at::Tensor wst;
  if (ws > 0) wst = at::empty({ws}, input.options().dtype(at::kByte));
  auto stream = at::cuda::getCurrentCUDAStream(input.device().index());
  check_status(b2g_pointwise_conv(x.data_ptr<float>(), wt.data_ptr<float>(), bp,
                                  out.data_ptr<float>(), bs, cin, cout, h * w, prec,
                                  ws > 0 ? wst.data_ptr() : nullptr, ws, stream.stream()),
               "b2g_pointwise_conv");
  return out;
}

// kernels/97_ScaledDotProductAttention_best_kernel.cu:256 (fused_attention_cuda) —
// out = softmax(Q K^T / sqrt(D)) V for fp16 (batch, heads, seq, dim) tensors.
at::Tensor fused_attention(at::Tensor Q, at::Tensor K, at::Tensor V) {
  for (const auto& t : {Q, K, V}) {
    TORCH_CHECK(t.is_cuda(), "Q, K and V must be CUDA tensors");
    TORCH_CHECK(t.scalar_type() == at::kHalf, "Q, K and V must be float16");
    TORCH_CHECK(t.dim() == 4, "Q, K and V must be (batch, heads, seq, dim)");
  }
  TORCH_CHECK(K.sizes() == Q.sizes() && V.sizes() == Q.sizes(), "Q, K and V must have one shape");
  TORCH_CHECK(K.device() == Q.device() && V.device() == Q.device(),
              "Q, K and V must be on the same device");
  const int64_t b = Q.size(0), h = Q.size(1), s = Q.size(2), d = Q.size(3);
  TORCH_CHECK(s <= 512, "Sequence length exceeds 512 (the score row is kept on chip).");
  TORCH_CHECK(d % 64 == 0, "Embedding dimension must be a multiple of 64.");
  const c10::cuda::CUDAGuard guard(Q.device());
  at::Tensor q = Q.contiguous(), k = K.contiguous(), v = V.contiguous();
  at::Tensor out = at::empty_like(q);
  if (out.numel() == 0) return out;
  auto stream = at::cuda::getCurrentCUDAStream(Q.device().index());
  check_status(b2g_sdpa(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), b, h, s, d,
                        0.f, stream.stream()),
               "b2g_sdpa");
  return out;
}

// Generic entry: op(A) . op(B) with explicit flags (used by the partitioner).
at::Tensor gemm(at::Tensor A, at::Tensor B, bool trans_a, bool trans_b, int64_t op) {
  return matmul_2d(trans_a ? A.t() : A, trans_b ? B.t() : B, static_cast<int>(op));
}

void set_precision(int64_t p) {
  TORCH_CHECK(p == B2G_PREC_TF32 || p == B2G_PREC_3XTF32, "precision must be 0 (tf32) or 1 (3xtf32)");
  g_precision.store(static_cast<int>(p));
}
int64_t get_precision() { return precision_now(); }
int64_t get_default_precision() { return g_precision.load(); }
// p = -1 removes this thread's override.
void set_thread_precision(int64_t p) {
  TORCH_CHECK(p == -1 || p == B2G_PREC_TF32 || p == B2G_PREC_3XTF32,
              "precision must be -1 (none), 0 (tf32) or 1 (3xtf32)");
  t_precision = static_cast<int>(p);
}
int64_t get_thread_precision() { return t_precision; }

// One epoch of the cross-GPU K-split sum on the current stream (the
// partitioner's per-step call; the same as b2g_splitk_peer_reduce through
// ctypes, without the per-call conversion cost).  t: the root's output
// (holding its own partial) or another rank's partial.
void splitk_peer_reduce(at::Tensor t, std::vector<int64_t> mailboxes, int64_t rank, int64_t root,
                        int64_t epoch) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kFloat && t.is_contiguous(),
              "peer reduce needs a contiguous CUDA float32 tensor");
  std::vector<void*> boxes(mailboxes.size());
  for (size_t r = 0; r < mailboxes.size(); ++r) boxes[r] = reinterpret_cast<void*>(mailboxes[r]);
  const c10::cuda::CUDAGuard guard(t.device());
  auto stream = at::cuda::getCurrentCUDAStream(t.device().index());
  float* p = t.data_ptr<float>();
  const bool is_root = rank == root;
  check_status(b2g_splitk_peer_reduce(is_root ? nullptr : p, is_root ? p : nullptr, t.numel(),
                                      boxes.data(), static_cast<int>(boxes.size()),
                                      static_cast<int>(rank), static_cast<int>(root), epoch,
                                      stream.stream()),
               "b2g_splitk_peer_reduce");
}

// This rank's K-slice product and the cross-GPU sum in one kernel
// (b2g_gemm_splitk_peer): A (M x K_r), B (K_r x N) this rank's slices, both
// row-major or transposed views; returns C (M x N), which on the root holds
// the full sum after the call and elsewhere this rank's partial.
at::Tensor splitk_peer_matmul(at::Tensor A, at::Tensor B, std::vector<int64_t> mailboxes,
                              int64_t rank, int64_t root, int64_t epoch) {
  check_input(A, "A");
  check_input(B, "B");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2, "A and B must be 2-D");
  TORCH_CHECK(A.device() == B.device(), "A and B must be on the same device");
  TORCH_CHECK(A.size(1) == B.size(0), "inner dimensions differ: A is ", A.sizes(), ", B is ",
              B.sizes());
  const c10::cuda::CUDAGuard guard(A.device());
  const int64_t M = A.size(0), K = A.size(1), N = B.size(1);
  at::Tensor C = at::empty({M, N}, A.options());
  if (M == 0 || N == 0) return C;
  Operand a = as_operand(A), b = as_operand(B);
  b2g_gemm_desc d{};
  d.op = B2G_OP_GEMM;
  d.precision = precision_now();
  d.m = M;
  d.n = N;
  d.k = K;
  d.batch = 1;
  d.a = a.ptr;
  d.lda = a.ld;
  d.trans_a = a.trans;
  d.b = b.ptr;
  d.ldb = b.ld;
  d.trans_b = b.trans;
  d.c = C.data_ptr<float>();
  d.ldc = N;
  const int64_t ws = b2g_gemm_workspace_bytes(&d);
  TORCH_CHECK(ws >= 0, "b2g: invalid GEMM descriptor");
  at::Tensor wst;
  if (ws > 0) {
    wst = at::empty({ws}, A.options().dtype(at::kByte));
    d.workspace = wst.data_ptr();
    d.workspace_bytes = ws;
  }
  std::vector<void*> boxes(mailboxes.size());
  for (size_t r = 0; r < mailboxes.size(); ++r) boxes[r] = reinterpret_cast<void*>(mailboxes[r]);
  auto stream = at::cuda::getCurrentCUDAStream(A.device().index());
  check_status(b2g_gemm_splitk_peer(&d, boxes.data(), static_cast<int>(boxes.size()),
                                    static_cast<int>(rank), static_cast<int>(root), epoch,
                                    stream.stream()),
               "b2g_gemm_splitk_peer");
  return C;
}

int64_t read_device_error(int64_t device) {
  int32_t code = 0;
  check_status(b2g_read_device_error(static_cast<int>(device), &code), "b2g_read_device_error");
  return code;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "B200 (sm_100a) fp32-input GEMM operator family";
  m.def("square_matmul", &square_matmul);
  m.def("standard_matmul", &standard_matmul);
  m.def("batched_matmul", &batched_matmul);
  m.def("batched_matmul_out", &batched_matmul_out, "C[b] = A[b] B[b] into a preallocated C");
  m.def("large_k_matmul", &large_k_matmul);
  m.def("small_k_matmul", &small_k_matmul);
  m.def("irregular_matmul", &irregular_matmul);
  m.def("tall_skinny_matmul", &tall_skinny_matmul);
  m.def("tensor3d_matmul", &tensor3d_matmul);
  m.def("tensor4d_matmul", &tensor4d_matmul);
  m.def("diag_matmul", &diag_matmul);
  m.def("symmetric_matmul", &symmetric_matmul);
  m.def("upper_tri_matmul", &upper_tri_matmul);
  m.def("lower_tri_matmul", &lower_tri_matmul);
  m.def("matmul_transposed_a", &matmul_transposed_a);
  m.def("matmul_transposed_b", &matmul_transposed_b);
  m.def("matmul_transposed_both", &matmul_transposed_both);
  m.def("gemv", &gemv);
  m.def("matrix_scalar_mult", &matrix_scalar_mult);
  m.def("fused_attention", &fused_attention, "softmax(Q K^T / sqrt(D)) V, fp16");
  m.def("pointwise_conv", &pointwise_conv_any, "1x1 convolution, NCHW", py::arg("input"),
        py::arg("weight"), py::arg("bias") = py::none());
  m.def("gemm", &gemm, "op(A) . op(B)", py::arg("A"), py::arg("B"), py::arg("trans_a") = false,
        py::arg("trans_b") = false, py::arg("op") = 0);
  m.def("set_precision", &set_precision);
  m.def("get_precision", &get_precision, "the mode this thread's calls use");
  m.def("get_default_precision", &get_default_precision);
  m.def("set_thread_precision", &set_thread_precision);
  m.def("get_thread_precision", &get_thread_precision);
  m.def("read_device_error", &read_device_error);
  m.def("splitk_peer_reduce", &splitk_peer_reduce, "one epoch of the cross-GPU K-split sum");
  m.def("splitk_peer_matmul", &splitk_peer_matmul,
        "this rank's K-slice product and the cross-GPU sum, one kernel");
}
