// PyTorch bindings: adapts torch tensors to the plain launch API in kernels.h.
// Every function checks devices, dtypes and contiguity and enqueues on the current stream.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstring>
#include <vector>

#include "attention.h"
#include "kernels.h"
#include "symm_comm.h"

namespace {

using torch::Tensor;

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void check_cuda(const Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), "mmf: ", name, " must be a CUDA tensor");
}
void check_bf16_contig(const Tensor& t, const char* name) {
  check_cuda(t, name);
  TORCH_CHECK(t.scalar_type() == torch::kBFloat16, "mmf: ", name, " must be bfloat16");
  TORCH_CHECK(t.is_contiguous(), "mmf: ", name, " must be contiguous");
}
const float* opt_f32_ptr(const c10::optional<Tensor>& t, const char* name) {
  if (!t.has_value()) return nullptr;
  check_cuda(*t, name);
  TORCH_CHECK(t->scalar_type() == torch::kFloat32 && t->is_contiguous(), "mmf: ", name, " must be contiguous fp32");
  return t->data_ptr<float>();
}

// Copy a vector of POD descriptors to the device through a pinned staging tensor.
template <typename T>
Tensor upload(const std::vector<T>& v, const torch::Device& dev) {
  const int64_t bytes = static_cast<int64_t>(v.size() * sizeof(T));
  Tensor host = torch::empty({bytes}, torch::dtype(torch::kUInt8).pinned_memory(true));
  std::memcpy(host.data_ptr(), v.data(), bytes);
  return host.to(dev, /*non_blocking=*/true);
}

Tensor ptr_table(const std::vector<Tensor>& ts) {
  TORCH_CHECK(!ts.empty(), "mmf: empty pointer table");
  std::vector<int64_t> ptrs;
  ptrs.reserve(ts.size());
  for (const auto& t : ts) {
    check_cuda(t, "tensor");
    ptrs.push_back(reinterpret_cast<int64_t>(t.data_ptr()));
  }
  Tensor host = torch::empty({static_cast<int64_t>(ptrs.size())}, torch::dtype(torch::kInt64).pinned_memory(true));
  std::memcpy(host.data_ptr(), ptrs.data(), ptrs.size() * sizeof(int64_t));
  return host.to(ts[0].device(), true);
}

void gemm_dims(const Tensor& A, const Tensor& B, bool b_mn, int& batch, int& M, int& N, int& K) {
  TORCH_CHECK(A.dim() == 3 && B.dim() == 3, "mmf: GEMM operands must be [batch, rows, cols]");
  batch = static_cast<int>(A.size(0));
  M = static_cast<int>(A.size(1));
  K = static_cast<int>(A.size(2));
  TORCH_CHECK(B.size(0) == batch, "mmf: batch mismatch");
  if (b_mn) {
    TORCH_CHECK(B.size(1) == K, "mmf: K mismatch (B is [batch, K, N])");
    N = static_cast<int>(B.size(2));
  } else {
    TORCH_CHECK(B.size(2) == K, "mmf: K mismatch (B is [batch, N, K])");
    N = static_cast<int>(B.size(1));
  }
}

void tc_gemm_ws(Tensor A, Tensor B, bool b_mn_major, Tensor D, c10::optional<Tensor> C,
                c10::optional<Tensor> alpha_vec, double alpha, c10::optional<Tensor> beta_vec, double beta,
                bool symmetric) {
  check_bf16_contig(A, "A");
  check_bf16_contig(B, "B");
  check_bf16_contig(D, "D");
  const c10::cuda::CUDAGuard guard(A.device());
  mmf::GemmWsArgs a{};
  gemm_dims(A, B, b_mn_major, a.batch, a.M, a.N, a.K);
  TORCH_CHECK(D.dim() == 3 && D.size(0) == a.batch && D.size(1) == a.M && D.size(2) == a.N, "mmf: D shape mismatch");
  if (C.has_value()) {
    check_bf16_contig(*C, "C");
    TORCH_CHECK(C->sizes() == D.sizes(), "mmf: C shape mismatch");
    TORCH_CHECK(C->data_ptr() != D.data_ptr(), "mmf: C must not alias D");
  }
  a.A = A.data_ptr();
  a.B = B.data_ptr();
  a.b_mn_major = b_mn_major;
  a.D = D.data_ptr();
  a.C = C.has_value() ? C->data_ptr() : nullptr;
  a.alpha_vec = opt_f32_ptr(alpha_vec, "alpha_vec");
  a.alpha = static_cast<float>(alpha);
  a.beta_vec = opt_f32_ptr(beta_vec, "beta_vec");
  a.beta = static_cast<float>(beta);
  a.symmetric = symmetric;
  mmf::tc_gemm_ws(a, cur_stream());
}

void tc_gemm_out(Tensor A, Tensor B, bool b_mn_major, c10::optional<Tensor> C, c10::optional<Tensor> alpha_vec,
                 double alpha, c10::optional<Tensor> beta_vec, double beta, Tensor out_ptrs, int64_t nseg,
                 c10::optional<Tensor> out_meta, int64_t out_ld,
                 bool out_f32, bool out_transposed, int64_t m_true, int64_t n_true, c10::optional<Tensor> p_scale_vec,
                 double p_scale, c10::optional<Tensor> v_scale_vec, double v_scale) {
  check_bf16_contig(A, "A");
  check_bf16_contig(B, "B");
  const c10::cuda::CUDAGuard guard(A.device());
  mmf::GemmOutArgs a{};
  gemm_dims(A, B, b_mn_major, a.batch, a.M, a.N, a.K);
  if (C.has_value()) {
    check_bf16_contig(*C, "C");
    TORCH_CHECK(C->dim() == 3 && C->size(0) == a.batch && C->size(1) == a.M && C->size(2) == a.N,
                "mmf: C shape mismatch");
  }
  check_cuda(out_ptrs, "out_ptrs");
  TORCH_CHECK(nseg >= 1, "mmf: nseg must be >= 1");
  TORCH_CHECK(out_ptrs.scalar_type() == torch::kInt64 && out_ptrs.numel() == a.batch * nseg,
              "mmf: out_ptrs must be int64[batch * nseg]");
  if (out_meta.has_value())
    TORCH_CHECK(out_meta->is_cuda() && out_meta->scalar_type() == torch::kInt64 && out_meta->numel() == 3 * a.batch,
                "mmf: out_meta must be a CUDA int64[batch * 3]");
  a.A = A.data_ptr();
  a.B = B.data_ptr();
  a.b_mn_major = b_mn_major;
  a.C = C.has_value() ? C->data_ptr() : nullptr;
  a.alpha_vec = opt_f32_ptr(alpha_vec, "alpha_vec");
  a.alpha = static_cast<float>(alpha);
  a.beta_vec = opt_f32_ptr(beta_vec, "beta_vec");
  a.beta = static_cast<float>(beta);
  a.out_ptrs = out_ptrs.data_ptr<int64_t>();
  a.nseg = static_cast<int>(nseg);
  a.out_meta = out_meta.has_value() ? out_meta->data_ptr<int64_t>() : nullptr;
  a.out_ld = out_ld;
  a.out_f32 = out_f32;
  a.out_transposed = out_transposed;
  a.m_true = static_cast<int>(m_true);
  a.n_true = static_cast<int>(n_true);
  a.p_scale_vec = opt_f32_ptr(p_scale_vec, "p_scale_vec");
  a.p_scale = static_cast<float>(p_scale);
  a.v_scale_vec = opt_f32_ptr(v_scale_vec, "v_scale_vec");
  a.v_scale = static_cast<float>(v_scale);
  mmf::tc_gemm_out(a, cur_stream());
}

// Weight gradient of a linear layer, scattered by rows: dW = dY^T X ([N, K] from dY [T, N] and
// X [T, K]), row r of dW goes to segment r / seg_rows (out_ptrs[seg], leading dimension and
// seg_rows from out_meta = [ld, 0, seg_rows] on the device); T = p_scale * T + dW + beta * C.
void wgrad_out(Tensor dY, Tensor X, Tensor out_ptrs, int64_t nseg, Tensor out_meta, bool out_f32, double p_scale,
               c10::optional<Tensor> C, double beta) {
  check_bf16_contig(dY, "dY");
  check_bf16_contig(X, "X");
  TORCH_CHECK(dY.dim() == 2 && X.dim() == 2 && dY.size(0) == X.size(0), "mmf: wgrad_out needs dY [T, N], X [T, K]");
  check_cuda(out_ptrs, "out_ptrs");
  TORCH_CHECK(out_ptrs.scalar_type() == torch::kInt64 && out_ptrs.numel() == nseg, "mmf: out_ptrs must be int64[nseg]");
  TORCH_CHECK(out_meta.is_cuda() && out_meta.scalar_type() == torch::kInt64 && out_meta.numel() == 3,
              "mmf: out_meta must be a CUDA int64[3]");
  const c10::cuda::CUDAGuard guard(dY.device());
  mmf::GemmOutArgs a{};
  a.A = dY.data_ptr();
  a.a_mn_major = true;
  a.B = X.data_ptr();
  a.b_mn_major = true;
  a.batch = 1;
  a.M = static_cast<int>(dY.size(1));
  a.N = static_cast<int>(X.size(1));
  a.K = static_cast<int>(dY.size(0));
  a.alpha = 1.f;
  a.beta = 0.f;
  if (C.has_value()) {  // + beta * C, C [N, K] bf16 (an unsharded gradient accumulator)
    check_bf16_contig(*C, "C");
    TORCH_CHECK(C->dim() == 2 && C->size(0) == a.M && C->size(1) == a.N, "mmf: wgrad_out: C must be [N, K]");
    a.C = C->data_ptr();
    a.beta = static_cast<float>(beta);
  }
  a.out_ptrs = out_ptrs.data_ptr<int64_t>();
  a.nseg = static_cast<int>(nseg);
  a.out_meta = out_meta.data_ptr<int64_t>();
  a.out_ld = 0;
  a.out_f32 = out_f32;
  a.m_true = a.M;
  a.n_true = a.N;
  a.p_scale = static_cast<float>(p_scale);
  a.v_scale = 1.f;
  mmf::tc_gemm_out(a, cur_stream());
}

// Grouped transformer-linear GEMM (linear_gemm.cu).  Shapes are read from the tensors:
//   forward         (a_mn=0, b_mn=0): A = [X [M, K]],        B = [W_s [N_s, K]],  out = [Y_s [M, N_s]]
//   input gradient  (a_mn=0, b_mn=1): A = [dY_s [M, K_s]],   B = [W_s [K_s, N]],  out = [dX [M, N]]
//   weight gradient (a_mn=1, b_mn=1): A = [dY_s [T, N_s]],   B = [X [T, K]],      out = [dW_s [N_s, K]]
// SWIGLU: B = [W1, W3] ([F, K] each), out = [h, g, u] ([M, F] each).  SWIGLU_BWD: out = [dg, du],
// aux0 = g, aux1 = u.  GELU: out = [gelu(z), z].  GELU_BWD: out = [dz], aux0 = z.
void linear_gemm(std::vector<Tensor> A, std::vector<Tensor> B, bool a_mn, bool b_mn, std::vector<Tensor> out,
                 int64_t epilogue, c10::optional<Tensor> C, c10::optional<Tensor> aux0, c10::optional<Tensor> aux1,
                 c10::optional<Tensor> bias, double alpha, bool accumulate, int64_t rope_mask, int64_t seq_len,
                 int64_t head_dim, double rope_theta) {
  TORCH_CHECK(!A.empty() && !B.empty() && !out.empty(), "mmf: linear_gemm needs operands and outputs");
  TORCH_CHECK(A.size() <= 3 && B.size() <= 3 && out.size() <= 3, "mmf: linear_gemm takes at most 3 segments");
  for (auto& t : A) check_bf16_contig(t, "A");
  for (auto& t : B) check_bf16_contig(t, "B");
  for (auto& t : A) TORCH_CHECK(t.dim() == 2, "mmf: linear_gemm operands are 2-D");
  for (auto& t : B) TORCH_CHECK(t.dim() == 2, "mmf: linear_gemm operands are 2-D");
  const auto dev = A[0].device();
  for (auto& t : out) {
    check_cuda(t, "out");
    TORCH_CHECK(t.device() == dev && t.dim() == 2 && t.is_contiguous(), "mmf: outputs must be contiguous 2-D on A's device");
    TORCH_CHECK(t.scalar_type() == out[0].scalar_type(), "mmf: outputs must share one dtype");
  }
  const bool f32 = out[0].scalar_type() == torch::kFloat32;
  TORCH_CHECK(f32 || out[0].scalar_type() == torch::kBFloat16, "mmf: outputs must be bf16 or fp32");
  const c10::cuda::CUDAGuard guard(dev);
  mmf::LinearGemmArgs a{};
  a.a_mn = a_mn;
  a.b_mn = b_mn;
  a.epilogue = static_cast<int>(epilogue);
  a.alpha = static_cast<float>(alpha);
  a.accumulate = accumulate;
  a.out_f32 = f32;
  const int na = static_cast<int>(A.size()), nb = static_cast<int>(B.size());
  for (int s = 0; s < na; ++s) {
    a.A[s] = A[s].data_ptr();
    a.a_outer[s] = A[s].size(0);
    a.a_inner[s] = A[s].size(1);
  }
  for (int s = 0; s < nb; ++s) {
    a.B[s] = B[s].data_ptr();
    a.b_outer[s] = B[s].size(0);
    a.b_inner[s] = B[s].size(1);
  }
  for (size_t s = 0; s < out.size(); ++s) {
    a.out[s] = out[s].data_ptr();
    a.ldo[s] = out[s].size(1);
  }
  if (!a_mn && !b_mn) {  // forward
    TORCH_CHECK(na == 1, "mmf: forward takes one input X");
    a.M = static_cast<int>(A[0].size(0));
    a.K[0] = static_cast<int>(A[0].size(1));
    for (int s = 0; s < nb; ++s) TORCH_CHECK(B[s].size(1) == a.K[0], "mmf: weight in-features mismatch");
    if (epilogue == mmf::LIN_EPI_SWIGLU) {
      TORCH_CHECK(nb == 2 && B[0].sizes() == B[1].sizes() && out.size() == 3, "mmf: SWIGLU takes W1, W3 -> h, g, u");
      a.axis = mmf::LIN_SEG_N;
      a.nseg = 2;
      a.N = static_cast<int>(B[0].size(0));
      for (auto& t : out) TORCH_CHECK(t.size(0) == a.M && t.size(1) == a.N, "mmf: SWIGLU outputs are [M, F]");
    } else if (epilogue == mmf::LIN_EPI_GELU) {
      TORCH_CHECK(nb == 1 && out.size() == 2, "mmf: GELU takes one weight -> gelu(z), z");
      a.axis = mmf::LIN_SEG_NONE;
      a.nseg = 1;
      a.N = static_cast<int>(B[0].size(0));
      for (auto& t : out) TORCH_CHECK(t.size(0) == a.M && t.size(1) == a.N, "mmf: GELU outputs are [M, N]");
    } else {
      TORCH_CHECK(static_cast<int>(out.size()) == nb, "mmf: one output per weight");
      a.axis = nb > 1 ? mmf::LIN_SEG_N : mmf::LIN_SEG_NONE;
      a.nseg = nb;
      a.N = 0;
      for (int s = 0; s < nb; ++s) {
        TORCH_CHECK(out[s].size(0) == a.M && out[s].size(1) == B[s].size(0), "mmf: output shape mismatch");
        a.seg_len[s] = static_cast<int>(B[s].size(0));
        a.N += a.seg_len[s];
      }
    }
  } else if (!a_mn && b_mn) {  // input gradient
    TORCH_CHECK(na == nb, "mmf: one weight per output gradient");
    a.M = static_cast<int>(A[0].size(0));
    a.N = static_cast<int>(B[0].size(1));
    for (int s = 0; s < na; ++s) {
      TORCH_CHECK(A[s].size(0) == a.M && B[s].size(1) == a.N && A[s].size(1) == B[s].size(0),
                  "mmf: input-gradient operand shapes mismatch");
      a.K[s] = static_cast<int>(A[s].size(1));
    }
    a.axis = na > 1 ? mmf::LIN_SEG_K : mmf::LIN_SEG_NONE;
    a.nseg = na;
    const size_t nout = epilogue == mmf::LIN_EPI_SWIGLU_BWD ? 2 : 1;
    TORCH_CHECK(out.size() == nout, "mmf: wrong number of outputs for this epilogue");
    for (auto& t : out) TORCH_CHECK(t.size(0) == a.M && t.size(1) == a.N, "mmf: output shape mismatch");
  } else {  // weight gradient
    TORCH_CHECK(a_mn && b_mn && nb == 1, "mmf: weight gradient takes dY segments and one X");
    TORCH_CHECK(static_cast<int>(out.size()) == na, "mmf: one weight gradient per dY segment");
    a.K[0] = static_cast<int>(B[0].size(0));
    a.N = static_cast<int>(B[0].size(1));
    a.M = 0;
    for (int s = 0; s < na; ++s) {
      TORCH_CHECK(A[s].size(0) == a.K[0], "mmf: dY and X token counts differ");
      TORCH_CHECK(out[s].size(0) == A[s].size(1) && out[s].size(1) == a.N, "mmf: weight-gradient shape mismatch");
      a.seg_len[s] = static_cast<int>(A[s].size(1));
      a.M += a.seg_len[s];
    }
    a.axis = na > 1 ? mmf::LIN_SEG_M : mmf::LIN_SEG_NONE;
    a.nseg = na;
  }
  if (C.has_value()) {
    check_bf16_contig(*C, "C");
    TORCH_CHECK(C->dim() == 2 && C->size(0) == a.M && C->size(1) == a.N, "mmf: C must be [M, N]");
    a.C = C->data_ptr();
    a.ldc = C->size(1);
  }
  if (aux0.has_value()) {
    check_bf16_contig(*aux0, "aux0");
    TORCH_CHECK(aux0->dim() == 2 && aux0->size(0) == a.M && aux0->size(1) == a.N, "mmf: aux0 must be [M, N]");
    a.aux0 = aux0->data_ptr();
    a.ld_aux = aux0->size(1);
  }
  if (aux1.has_value()) {
    check_bf16_contig(*aux1, "aux1");
    TORCH_CHECK(aux1->sizes() == aux0->sizes(), "mmf: aux1 must match aux0");
    a.aux1 = aux1->data_ptr();
  }
  if (bias.has_value()) {
    check_bf16_contig(*bias, "bias");
    TORCH_CHECK(bias->numel() == a.N, "mmf: bias must have N elements");
    a.bias = bias->data_ptr();
  }
  a.rope_mask = static_cast<int>(rope_mask);
  a.seq_len = static_cast<int>(seq_len);
  a.head_dim = static_cast<int>(head_dim);
  a.rope_theta = static_cast<float>(rope_theta);
  mmf::linear_gemm(a, cur_stream());
}

// GEMM -> reduce-scatter, first half: dW = dY^T X (+ C, an unsharded gradient accumulator),
// row r stored to owner_ptrs[r / rows_per_owner] + ((r % rows_per_owner) * K + col) elements
// (owner_ptrs: device int64 table, e.g. this rank's sub-slot in every owner's receive buffer).
void wgrad_scatter(Tensor dY, Tensor X, Tensor owner_ptrs, int64_t rows_per_owner, c10::optional<Tensor> C) {
  check_bf16_contig(dY, "dY");
  check_bf16_contig(X, "X");
  check_cuda(owner_ptrs, "owner_ptrs");
  TORCH_CHECK(dY.dim() == 2 && X.dim() == 2 && dY.size(0) == X.size(0), "mmf: wgrad_scatter needs dY [T, N], X [T, K]");
  TORCH_CHECK(owner_ptrs.scalar_type() == torch::kInt64 && owner_ptrs.is_contiguous(), "mmf: owner_ptrs must be int64");
  TORCH_CHECK(rows_per_owner >= 1 && owner_ptrs.numel() * rows_per_owner >= dY.size(1),
              "mmf: the owner table does not cover every output row");
  const c10::cuda::CUDAGuard guard(dY.device());
  mmf::LinearGemmArgs a{};
  a.a_mn = true;
  a.b_mn = true;
  a.epilogue = mmf::LIN_EPI_SCATTER;
  a.alpha = 1.f;
  a.axis = mmf::LIN_SEG_NONE;
  a.nseg = 1;
  a.A[0] = dY.data_ptr();
  a.a_outer[0] = dY.size(0);
  a.a_inner[0] = dY.size(1);
  a.B[0] = X.data_ptr();
  a.b_outer[0] = X.size(0);
  a.b_inner[0] = X.size(1);
  a.K[0] = static_cast<int>(dY.size(0));
  a.M = static_cast<int>(dY.size(1));
  a.N = static_cast<int>(X.size(1));
  a.ldo[0] = X.size(1);
  if (C.has_value()) {
    check_bf16_contig(*C, "C");
    TORCH_CHECK(C->dim() == 2 && C->size(0) == a.M && C->size(1) == a.N, "mmf: C must be [N, K]");
    a.C = C->data_ptr();
    a.ldc = a.N;
  }
  a.scatter_ptrs = owner_ptrs.data_ptr<int64_t>();
  a.scatter_nseg = static_cast<int>(owner_ptrs.numel());
  a.scatter_rows = rows_per_owner;
  mmf::linear_gemm(a, cur_stream());
}

// Y = X @ W^T with W row-sharded over the group (shard_ptrs: every rank's shard address in this
// process's address space); also assembles the full W into G.  ready: int32 [N / 128] scratch.
Tensor ag_gemm(Tensor X, std::vector<int64_t> shard_ptrs, int64_t rank, Tensor G, Tensor ready, double wait_s) {
  check_bf16_contig(X, "X");
  check_bf16_contig(G, "G");
  check_cuda(ready, "ready");
  TORCH_CHECK(X.dim() == 2 && G.dim() == 2 && X.size(1) == G.size(1), "mmf: ag_gemm needs X [M, K], G [N, K]");
  TORCH_CHECK(ready.scalar_type() == torch::kInt32 && ready.numel() >= G.size(0) / 128, "mmf: ready must be int32[N/128]");
  const int ws = static_cast<int>(shard_ptrs.size());
  TORCH_CHECK(ws >= 1 && ws <= 8, "mmf: ag_gemm supports 1..8 ranks");
  const c10::cuda::CUDAGuard guard(X.device());
  Tensor Y = torch::empty({X.size(0), G.size(0)}, X.options());
  mmf::AgGemmArgs a{};
  a.X = X.data_ptr();
  a.M = static_cast<int>(X.size(0));
  a.N = static_cast<int>(G.size(0));
  a.K = static_cast<int>(X.size(1));
  a.rank = static_cast<int>(rank);
  a.ws = ws;
  for (int s = 0; s < ws; ++s) a.shard_ptrs[s] = shard_ptrs[s];
  a.G = G.data_ptr();
  a.Y = Y.data_ptr();
  a.ready = reinterpret_cast<uint32_t*>(ready.data_ptr<int32_t>());
  a.wait_ns = static_cast<uint64_t>(wait_s * 1e9);
  mmf::ag_gemm(a, cur_stream());
  return Y;
}

// out (bf16, n elements) = (accumulate ? out : 0) + scale * sum over ranks s of
// slots[s * slot_stride : s * slot_stride + n] (rank order, fp32)
void rs_reduce(Tensor slots, int64_t ws, int64_t slot_stride, Tensor out, bool accumulate, double scale) {
  check_bf16_contig(slots, "slots");
  check_bf16_contig(out, "out");
  TORCH_CHECK(slot_stride >= out.numel() && slots.numel() >= (ws - 1) * slot_stride + out.numel(),
              "mmf: rs_reduce: slots too small");
  const c10::cuda::CUDAGuard guard(out.device());
  mmf::rs_reduce(slots.data_ptr(), static_cast<int>(ws), slot_stride, out.numel(), out.data_ptr(), accumulate,
                 static_cast<float>(scale), cur_stream());
}

// out (bf16) = (accumulate ? out : 0) + scale * sum over ranks s of srcs[s][offset : offset + numel(out)]
// (srcs: device int64 [ws] of every rank's partial buffer; P2P loads for the peers)
void rs_pull_reduce(Tensor srcs, int64_t offset, Tensor out, bool accumulate, double scale) {
  check_cuda(srcs, "srcs");
  check_bf16_contig(out, "out");
  TORCH_CHECK(srcs.scalar_type() == torch::kInt64, "mmf: srcs must be int64");
  const c10::cuda::CUDAGuard guard(out.device());
  mmf::rs_pull_reduce(srcs.data_ptr<int64_t>(), static_cast<int>(srcs.numel()), offset, out.numel(), out.data_ptr(),
                      accumulate, static_cast<float>(scale), cur_stream());
}

// grads/bufs/params: per-matrix tensors (bufs/params may be empty lists).  dst: optional bf16
// workspace; per-matrix destination = dst_base_offsets[i] elements into dst.
void muon_prep(std::vector<Tensor> grads, std::vector<Tensor> bufs, std::vector<Tensor> params,
               c10::optional<Tensor> dst, std::vector<int64_t> dst_offsets, std::vector<int64_t> dst_row0,
               std::vector<int64_t> transposed, std::vector<int64_t> dst_ld, std::vector<double> p_scale,
               std::vector<double> v_scale, int64_t mode, bool nesterov, double mu, double wd_coupled,
               c10::optional<Tensor> sumsq) {
  const int n = static_cast<int>(grads.size());
  if (n == 0) return;
  const auto dev = grads[0].device();
  const c10::cuda::CUDAGuard guard(dev);
  TORCH_CHECK(bufs.empty() || (int)bufs.size() == n, "mmf: bufs size");
  TORCH_CHECK(params.empty() || (int)params.size() == n, "mmf: params size");
  const bool grad_f32 = grads[0].scalar_type() == torch::kFloat32;
  const bool param_f32 = !params.empty() && params[0].scalar_type() == torch::kFloat32;
  if (dst.has_value()) {
    TORCH_CHECK((int)dst_offsets.size() == n && (int)dst_row0.size() == n && (int)transposed.size() == n &&
                    (dst_ld.size() == 1 || (int)dst_ld.size() == n),
                "mmf: per-tensor destination lists must match the number of tensors");
  } else {
    TORCH_CHECK((int)p_scale.size() == n && (int)v_scale.size() == n, "mmf: per-tensor scale lists size");
  }
  std::vector<mmf::PrepDesc> d(n);
  int max_tiles = 1;
  bool vec8 = true;
  for (int i = 0; i < n; ++i) {
    const Tensor& g = grads[i];
    check_cuda(g, "grad");
    TORCH_CHECK(g.is_contiguous() && g.dim() == 2, "mmf: grads must be contiguous 2-D");
    TORCH_CHECK((g.scalar_type() == torch::kFloat32) == grad_f32 &&
                    (g.scalar_type() == torch::kFloat32 || g.scalar_type() == torch::kBFloat16),
                "mmf: grads must all be fp32 or all bf16");
    d[i].grad = reinterpret_cast<int64_t>(g.data_ptr());
    d[i].rows = static_cast<int32_t>(g.size(0));
    d[i].cols = static_cast<int32_t>(g.size(1));
    if (!bufs.empty()) {
      TORCH_CHECK(bufs[i].scalar_type() == torch::kFloat32 && bufs[i].is_contiguous() && bufs[i].numel() == g.numel(),
                  "mmf: momentum buffers must be contiguous fp32 of the grad's size");
      d[i].buf = reinterpret_cast<int64_t>(bufs[i].data_ptr());
    }
    if (!params.empty()) {
      TORCH_CHECK(params[i].is_contiguous() && params[i].numel() == g.numel() &&
                      (params[i].scalar_type() == torch::kFloat32) == param_f32,
                  "mmf: params must be contiguous, same size, same dtype");
      d[i].param = reinterpret_cast<int64_t>(params[i].data_ptr());
    }
    if (dst.has_value()) {
      d[i].dst = reinterpret_cast<int64_t>(dst->data_ptr()) + dst_offsets[i] * 2;
      d[i].dst_row0 = static_cast<int32_t>(dst_row0[i]);
      d[i].transposed = static_cast<int32_t>(transposed[i]);
      d[i].dst_ld = dst_ld.size() == 1 ? dst_ld[0] : dst_ld[i];
    } else {
      TORCH_CHECK(!params.empty(), "mmf: direct apply needs params");
      d[i].p_scale = static_cast<float>(p_scale[i]);
      d[i].v_scale = static_cast<float>(v_scale[i]);
    }
    const int tiles = ((d[i].rows + 63) / 64) * ((d[i].cols + 63) / 64);
    if (tiles > max_tiles) max_tiles = tiles;
    auto al16 = [](int64_t p) { return (p & 15) == 0; };
    bool v = (d[i].cols % 8 == 0) && al16(d[i].grad) && al16(d[i].buf) && al16(d[i].param);
    if (dst.has_value()) v = v && al16(d[i].dst) && (d[i].dst_ld % 8 == 0) && (d[i].dst_row0 % 8 == 0);
    if (!v) vec8 = false;
  }
  if (mode != 0) {
    TORCH_CHECK(!bufs.empty(), "mmf: momentum modes need buffers");
  }
  if (dst.has_value()) check_bf16_contig(*dst, "dst");
  Tensor dd = upload(d, dev);
  mmf::PrepArgs a{};
  a.descs = reinterpret_cast<const mmf::PrepDesc*>(dd.data_ptr());
  a.n = n;
  a.max_tiles = max_tiles;
  a.grad_f32 = grad_f32;
  a.param_f32 = param_f32;
  a.mode = static_cast<int>(mode);
  a.nesterov = nesterov ? 1 : 0;
  a.mu = static_cast<float>(mu);
  a.wd_coupled = static_cast<float>(wd_coupled);
  a.sumsq = sumsq.has_value() ? sumsq->data_ptr<float>() : nullptr;
  Tensor partials;
  if (a.sumsq) {
    partials = torch::empty({static_cast<int64_t>(n) * mmf::muon_prep_blocks(max_tiles)},
                            torch::dtype(torch::kFloat32).device(dev));
    a.partials = partials.data_ptr<float>();
  }
  a.vec8 = vec8 ? 1 : 0;
  mmf::muon_prep(a, cur_stream());
}

void ns_scale(Tensor sumsq, int64_t n, int64_t nparts, double eps, Tensor s, c10::optional<Tensor> s2) {
  check_cuda(sumsq, "sumsq");
  const c10::cuda::CUDAGuard guard(sumsq.device());
  mmf::ns_scale(sumsq.data_ptr<float>(), static_cast<int>(n), static_cast<int>(nparts), static_cast<float>(eps),
                s.data_ptr<float>(), s2.has_value() ? s2->data_ptr<float>() : nullptr, cur_stream());
}

void ws_to_out(Tensor X, c10::optional<Tensor> s_vec, Tensor out_ptrs, int64_t nseg, c10::optional<Tensor> out_meta,
               int64_t out_ld, bool out_f32,
               bool out_transposed, int64_t m_true, int64_t n_true, c10::optional<Tensor> p_scale_vec, double p_scale,
               c10::optional<Tensor> v_scale_vec, double v_scale) {
  check_bf16_contig(X, "X");
  const c10::cuda::CUDAGuard guard(X.device());
  mmf::WsOutArgs a{};
  a.X = X.data_ptr();
  a.batch = static_cast<int>(X.size(0));
  a.Mp = static_cast<int>(X.size(1));
  a.Np = static_cast<int>(X.size(2));
  a.s_vec = opt_f32_ptr(s_vec, "s_vec");
  TORCH_CHECK(nseg >= 1 && out_ptrs.numel() == a.batch * nseg, "mmf: out_ptrs must be int64[batch * nseg]");
  a.out_ptrs = out_ptrs.data_ptr<int64_t>();
  a.nseg = static_cast<int>(nseg);
  a.out_meta = out_meta.has_value() ? out_meta->data_ptr<int64_t>() : nullptr;
  a.out_ld = out_ld;
  a.out_f32 = out_f32;
  a.out_transposed = out_transposed;
  a.m_true = static_cast<int>(m_true);
  a.n_true = static_cast<int>(n_true);
  a.p_scale_vec = opt_f32_ptr(p_scale_vec, "p_scale_vec");
  a.p_scale = static_cast<float>(p_scale);
  a.v_scale_vec = opt_f32_ptr(v_scale_vec, "v_scale_vec");
  a.v_scale = static_cast<float>(v_scale);
  mmf::ws_to_out(a, cur_stream());
}

// Per-tensor descriptors of a multi-tensor optimizer launch: params and grads of one dtype each
// (fp32 or bf16), two fp32 state tensors per param.  Returns the uploaded table.
struct OptDescs {
  Tensor table;
  int n = 0;
  int64_t max_numel = 1;
  bool p32 = false, g32 = false, vec4 = true;
};

OptDescs opt_descs(const std::vector<Tensor>& params, const std::vector<Tensor>& grads,
                   const std::vector<Tensor>& st_a, const std::vector<Tensor>& st_b, const char* what) {
  OptDescs o;
  o.n = static_cast<int>(params.size());
  const auto dev = params[0].device();
  TORCH_CHECK((int)grads.size() == o.n && (int)st_a.size() == o.n && (int)st_b.size() == o.n, "mmf: ", what,
              " list sizes differ");
  o.p32 = params[0].scalar_type() == torch::kFloat32;
  o.g32 = grads[0].scalar_type() == torch::kFloat32;
  std::vector<mmf::AdamDesc> d(o.n);
  for (int i = 0; i < o.n; ++i) {
    TORCH_CHECK(params[i].is_cuda() && params[i].is_contiguous() && grads[i].is_contiguous() &&
                    st_a[i].is_contiguous() && st_b[i].is_contiguous(),
                "mmf: ", what, " tensors must be contiguous CUDA tensors");
    TORCH_CHECK(params[i].device() == dev && grads[i].device() == dev && st_a[i].device() == dev &&
                    st_b[i].device() == dev,
                "mmf: ", what, " tensors must be on one device");
    TORCH_CHECK((params[i].scalar_type() == torch::kFloat32) == o.p32 &&
                    (grads[i].scalar_type() == torch::kFloat32) == o.g32,
                "mmf: ", what, " dtypes must be uniform within a launch");
    TORCH_CHECK(params[i].scalar_type() == torch::kFloat32 || params[i].scalar_type() == torch::kBFloat16,
                "mmf: ", what, " params must be fp32 or bf16");
    TORCH_CHECK(grads[i].scalar_type() == torch::kFloat32 || grads[i].scalar_type() == torch::kBFloat16,
                "mmf: ", what, " grads must be fp32 or bf16");
    TORCH_CHECK(st_a[i].scalar_type() == torch::kFloat32 && st_b[i].scalar_type() == torch::kFloat32,
                "mmf: ", what, " state tensors must be fp32");
    TORCH_CHECK(grads[i].numel() == params[i].numel() && st_a[i].numel() == params[i].numel() &&
                    st_b[i].numel() == params[i].numel(),
                "mmf: ", what, " sizes differ");
    d[i].param = reinterpret_cast<int64_t>(params[i].data_ptr());
    d[i].grad = reinterpret_cast<int64_t>(grads[i].data_ptr());
    d[i].exp_avg = reinterpret_cast<int64_t>(st_a[i].data_ptr());
    d[i].exp_avg_sq = reinterpret_cast<int64_t>(st_b[i].data_ptr());
    d[i].numel = params[i].numel();
    if (d[i].numel > o.max_numel) o.max_numel = d[i].numel;
    auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    if (d[i].numel % 4 != 0 || !al(params[i].data_ptr()) || !al(grads[i].data_ptr()) || !al(st_a[i].data_ptr()) ||
        !al(st_b[i].data_ptr()))
      o.vec4 = false;
  }
  o.table = upload(d, dev);
  return o;
}

void adamw(std::vector<Tensor> params, std::vector<Tensor> grads, std::vector<Tensor> exp_avgs,
           std::vector<Tensor> exp_avg_sqs, double lr, double beta1, double beta2, double eps, double weight_decay,
           double bias_correction1, double bias_correction2_sqrt) {
  if (params.empty()) return;
  const c10::cuda::CUDAGuard guard(params[0].device());
  OptDescs o = opt_descs(params, grads, exp_avgs, exp_avg_sqs, "adamw");
  mmf::AdamArgs a{};
  a.descs = reinterpret_cast<const mmf::AdamDesc*>(o.table.data_ptr());
  a.n = o.n;
  a.max_numel = o.max_numel;
  a.param_f32 = o.p32;
  a.grad_f32 = o.g32;
  a.lr = static_cast<float>(lr);
  a.beta1 = static_cast<float>(beta1);
  a.beta2 = static_cast<float>(beta2);
  a.eps = static_cast<float>(eps);
  a.weight_decay = static_cast<float>(weight_decay);
  a.bias_correction1 = static_cast<float>(bias_correction1);
  a.bias_correction2_sqrt = static_cast<float>(bias_correction2_sqrt);
  a.vec4 = o.vec4 ? 1 : 0;
  mmf::adamw_multi(a, cur_stream());
}

void muon_moments(std::vector<Tensor> params, std::vector<Tensor> grads, std::vector<Tensor> bufs,
                  std::vector<Tensor> second_moments, double momentum, double beta2, double weight_decay,
                  bool nesterov) {
  if (params.empty()) return;
  const c10::cuda::CUDAGuard guard(params[0].device());
  OptDescs o = opt_descs(params, grads, bufs, second_moments, "muon_moments");
  mmf::MomentArgs a{};
  a.descs = reinterpret_cast<const mmf::AdamDesc*>(o.table.data_ptr());
  a.n = o.n;
  a.max_numel = o.max_numel;
  a.param_f32 = o.p32;
  a.grad_f32 = o.g32;
  a.momentum = static_cast<float>(momentum);
  a.beta2 = static_cast<float>(beta2);
  a.weight_decay = static_cast<float>(weight_decay);
  a.nesterov = nesterov ? 1 : 0;
  a.vec4 = o.vec4 ? 1 : 0;
  mmf::muon_moments_multi(a, cur_stream());
}

// --------------------------------- model ops --------------------------------------------
std::vector<Tensor> rmsnorm_fwd(Tensor x, Tensor w, double eps) {
  check_bf16_contig(x, "x");
  check_bf16_contig(w, "w");
  const c10::cuda::CUDAGuard guard(x.device());
  const int cols = static_cast<int>(x.size(-1));
  const int rows = static_cast<int>(x.numel() / cols);
  TORCH_CHECK(w.numel() == cols, "mmf: rmsnorm weight size");
  Tensor y = torch::empty_like(x);
  Tensor rstd = torch::empty({rows}, x.options().dtype(torch::kFloat32));
  mmf::rmsnorm_fwd(x.data_ptr(), w.data_ptr(), y.data_ptr(), rstd.data_ptr<float>(), rows, cols,
                   static_cast<float>(eps), cur_stream());
  return {y, rstd};
}

std::vector<Tensor> rmsnorm_bwd(Tensor dy, Tensor x, Tensor w, Tensor rstd) {
  check_bf16_contig(dy, "dy");
  check_bf16_contig(x, "x");
  const c10::cuda::CUDAGuard guard(x.device());
  const int cols = static_cast<int>(x.size(-1));
  const int rows = static_cast<int>(x.numel() / cols);
  const int prow = std::max(1, std::min(rows, 296));
  Tensor dx = torch::empty_like(x);
  Tensor part = torch::empty({prow, cols}, x.options().dtype(torch::kFloat32));
  Tensor dw = torch::empty({cols}, w.options());
  mmf::rmsnorm_bwd(dy.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr<float>(), dx.data_ptr(),
                   part.data_ptr<float>(), rows, cols, prow, cur_stream());
  mmf::colsum_partials(part.data_ptr<float>(), prow, cols, dw.data_ptr(), w.scalar_type() == torch::kFloat32,
                       cur_stream());
  return {dx, dw};
}

// x *= s (bf16 x in place; s a one-element fp32 CUDA tensor, read on the device)
void scale_(Tensor x, Tensor s) {
  check_bf16_contig(x, "x");
  check_cuda(s, "s");
  TORCH_CHECK(s.scalar_type() == torch::kFloat32 && s.numel() == 1, "mmf: scale_ takes a one-element fp32 scale");
  const c10::cuda::CUDAGuard guard(x.device());
  mmf::scale_bf16(x.data_ptr(), s.data_ptr<float>(), x.numel(), cur_stream());
}

// out[..., :] = table[tokens[...]]   (table [V, D] bf16, tokens int64)
Tensor embedding_fwd(Tensor table, Tensor tokens) {
  check_bf16_contig(table, "table");
  check_cuda(tokens, "tokens");
  TORCH_CHECK(table.dim() == 2 && tokens.scalar_type() == torch::kInt64, "mmf: embedding takes a [V, D] table, int64 tokens");
  const c10::cuda::CUDAGuard guard(table.device());
  Tensor tok = tokens.contiguous();
  auto shape = tok.sizes().vec();
  shape.push_back(table.size(1));
  Tensor out = torch::empty(shape, table.options());
  mmf::embedding_fwd(table.data_ptr(), tok.data_ptr<int64_t>(), out.data_ptr(), tok.numel(),
                     static_cast<int>(table.size(1)), table.size(0), cur_stream());
  return out;
}

// Dense gradient of the table: row v = sum of dy over the positions whose token is v (fp32, in
// a fixed order), zeros elsewhere.  The token sort is a library sort of the (small) token list.
Tensor embedding_bwd(Tensor dy, Tensor tokens, int64_t vocab) {
  check_bf16_contig(dy, "dy");
  check_cuda(tokens, "tokens");
  const c10::cuda::CUDAGuard guard(dy.device());
  const int64_t D = dy.size(-1);
  Tensor tok = tokens.reshape({-1});
  TORCH_CHECK(tok.numel() * D == dy.numel(), "mmf: embedding_bwd: dy must be [..., D] over the tokens");
  auto sorted = torch::sort(tok, /*stable=*/true, /*dim=*/0, /*descending=*/false);
  Tensor s_tok = std::get<0>(sorted).contiguous();
  Tensor perm = std::get<1>(sorted).contiguous();
  Tensor first = torch::empty({vocab}, dy.options().dtype(torch::kInt32));
  Tensor dtable = torch::empty({vocab, D}, dy.options());
  mmf::embedding_bwd(dy.data_ptr(), s_tok.data_ptr<int64_t>(), perm.data_ptr<int64_t>(), first.data_ptr<int>(),
                     dtable.data_ptr(), tok.numel(), vocab, static_cast<int>(D), cur_stream());
  return dtable;
}

std::vector<Tensor> layernorm_fwd(Tensor x, Tensor w, c10::optional<Tensor> b, double eps) {
  check_bf16_contig(x, "x");
  check_bf16_contig(w, "w");
  const c10::cuda::CUDAGuard guard(x.device());
  const int cols = static_cast<int>(x.size(-1));
  const int rows = static_cast<int>(x.numel() / cols);
  Tensor y = torch::empty_like(x);
  Tensor mean = torch::empty({rows}, x.options().dtype(torch::kFloat32));
  Tensor rstd = torch::empty({rows}, x.options().dtype(torch::kFloat32));
  mmf::layernorm_fwd(x.data_ptr(), w.data_ptr(), b.has_value() ? b->data_ptr() : nullptr, y.data_ptr(),
                     mean.data_ptr<float>(), rstd.data_ptr<float>(), rows, cols, static_cast<float>(eps), cur_stream());
  return {y, mean, rstd};
}

std::vector<Tensor> layernorm_bwd(Tensor dy, Tensor x, Tensor w, Tensor mean, Tensor rstd, bool has_bias) {
  check_bf16_contig(dy, "dy");
  check_bf16_contig(x, "x");
  const c10::cuda::CUDAGuard guard(x.device());
  const int cols = static_cast<int>(x.size(-1));
  const int rows = static_cast<int>(x.numel() / cols);
  const int prow = std::max(1, std::min(rows, 296));
  Tensor dx = torch::empty_like(x);
  Tensor pw = torch::empty({prow, cols}, x.options().dtype(torch::kFloat32));
  Tensor pb = torch::empty({prow, cols}, x.options().dtype(torch::kFloat32));
  mmf::layernorm_bwd(dy.data_ptr(), x.data_ptr(), w.data_ptr(), mean.data_ptr<float>(), rstd.data_ptr<float>(),
                     dx.data_ptr(), pw.data_ptr<float>(), pb.data_ptr<float>(), rows, cols, prow, cur_stream());
  Tensor dw = torch::empty({cols}, w.options());
  mmf::colsum_partials(pw.data_ptr<float>(), prow, cols, dw.data_ptr(), w.scalar_type() == torch::kFloat32,
                       cur_stream());
  Tensor db;
  if (has_bias) {
    db = torch::empty({cols}, w.options());
    mmf::colsum_partials(pb.data_ptr<float>(), prow, cols, db.data_ptr(), w.scalar_type() == torch::kFloat32,
                         cur_stream());
  }
  return {dx, dw, db};
}

// x viewed as [tokens, heads, head_dim] with arbitrary token/head strides (elements).
void rope_(Tensor x, int64_t tokens, int64_t heads, int64_t head_dim, int64_t seq_len, double theta, bool inverse,
           int64_t token_stride, int64_t head_stride) {
  check_cuda(x, "x");
  TORCH_CHECK(x.scalar_type() == torch::kBFloat16, "mmf: rope input must be bf16");
  const c10::cuda::CUDAGuard guard(x.device());
  mmf::rope_inplace(x.data_ptr(), static_cast<int>(tokens), static_cast<int>(heads), static_cast<int>(head_dim),
                    static_cast<int>(seq_len), static_cast<float>(theta), inverse, token_stride, head_stride,
                    cur_stream());
}

Tensor swiglu_fwd(Tensor g, Tensor u) {
  check_bf16_contig(g, "gate");
  check_bf16_contig(u, "up");
  const c10::cuda::CUDAGuard guard(g.device());
  Tensor o = torch::empty_like(g);
  mmf::swiglu_fwd(g.data_ptr(), u.data_ptr(), o.data_ptr(), g.numel(), cur_stream());
  return o;
}
std::vector<Tensor> swiglu_bwd(Tensor d, Tensor g, Tensor u) {
  check_bf16_contig(d, "dout");
  const c10::cuda::CUDAGuard guard(g.device());
  Tensor dg = torch::empty_like(g), du = torch::empty_like(u);
  mmf::swiglu_bwd(d.data_ptr(), g.data_ptr(), u.data_ptr(), dg.data_ptr(), du.data_ptr(), g.numel(), cur_stream());
  return {dg, du};
}
Tensor gelu_fwd(Tensor x) {
  check_bf16_contig(x, "x");
  const c10::cuda::CUDAGuard guard(x.device());
  Tensor y = torch::empty_like(x);
  mmf::gelu_fwd(x.data_ptr(), y.data_ptr(), x.numel(), cur_stream());
  return y;
}
Tensor gelu_bwd(Tensor dy, Tensor x) {
  check_bf16_contig(dy, "dy");
  const c10::cuda::CUDAGuard guard(x.device());
  Tensor dx = torch::empty_like(x);
  mmf::gelu_bwd(dy.data_ptr(), x.data_ptr(), dx.data_ptr(), x.numel(), cur_stream());
  return dx;
}

// logits [rows, >=vocab] bf16 (row stride ld), targets int64 [rows]. Returns per-row loss.
Tensor cross_entropy_(Tensor logits, Tensor targets, int64_t vocab, double grad_scale, int64_t ignore_index) {
  check_cuda(logits, "logits");
  TORCH_CHECK(logits.scalar_type() == torch::kBFloat16 && logits.dim() == 2 && logits.stride(1) == 1,
              "mmf: logits must be bf16 [rows, vocab] with unit column stride");
  TORCH_CHECK(targets.scalar_type() == torch::kInt64 && targets.is_contiguous(), "mmf: targets must be int64");
  const c10::cuda::CUDAGuard guard(logits.device());
  const int rows = static_cast<int>(logits.size(0));
  Tensor loss = torch::empty({rows}, logits.options().dtype(torch::kFloat32));
  mmf::cross_entropy_fwd_bwd(logits.data_ptr(), targets.data_ptr<int64_t>(), loss.data_ptr<float>(), rows,
                             static_cast<int>(vocab), logits.stride(0), static_cast<float>(grad_scale),
                             static_cast<int>(ignore_index), cur_stream());
  return loss;
}

void power_iteration(Tensor W, Tensor u, Tensor v, Tensor sigma, int64_t iters, double eps, Tensor work) {
  check_cuda(W, "W");
  TORCH_CHECK(W.dim() == 2 && W.is_contiguous(), "mmf: W must be contiguous 2-D");
  TORCH_CHECK(W.scalar_type() == torch::kFloat32 || W.scalar_type() == torch::kBFloat16, "mmf: W dtype");
  const c10::cuda::CUDAGuard guard(W.device());
  TORCH_CHECK(work.numel() >= std::max(W.size(0), W.size(1)) + 1, "mmf: work too small");
  Tensor col_part = torch::empty({static_cast<int64_t>(mmf::power_iteration_col_blocks(static_cast<int>(W.size(0)))) *
                                      W.size(1)},
                                 torch::dtype(torch::kFloat32).device(W.device()));
  mmf::power_iteration(W.data_ptr(), W.scalar_type() == torch::kFloat32, static_cast<int>(W.size(0)),
                       static_cast<int>(W.size(1)), u.data_ptr<float>(), v.data_ptr<float>(), sigma.data_ptr<float>(),
                       static_cast<int>(iters), static_cast<float>(eps), work.data_ptr<float>(),
                       col_part.data_ptr<float>(), cur_stream());
}

// pad_ptrs / payload_ptrs: device int64 tensors of per-rank addresses (symmetric memory).
void symm_barrier(Tensor pad_ptrs, int64_t rank, int64_t ws, int64_t epoch, int64_t slot_base,
                  c10::optional<Tensor> payload, c10::optional<Tensor> payload_ptrs, double timeout_s) {
  check_cuda(pad_ptrs, "pad_ptrs");
  TORCH_CHECK(pad_ptrs.scalar_type() == torch::kInt64 && pad_ptrs.numel() == ws, "mmf: pad_ptrs must be int64[ws]");
  const float* pl = nullptr;
  int n = 0;
  const int64_t* pp = nullptr;
  if (payload.has_value()) {
    TORCH_CHECK(payload_ptrs.has_value() && payload_ptrs->numel() == ws, "mmf: payload needs payload_ptrs[ws]");
    TORCH_CHECK(payload->scalar_type() == torch::kFloat32 && payload->is_contiguous(), "mmf: payload must be fp32");
    pl = payload->data_ptr<float>();
    n = static_cast<int>(payload->numel());
    pp = payload_ptrs->data_ptr<int64_t>();
  }
  const c10::cuda::CUDAGuard guard(pad_ptrs.device());
  mmf::symm_barrier(pad_ptrs.data_ptr<int64_t>(), static_cast<int>(rank), static_cast<int>(ws),
                    static_cast<uint32_t>(epoch), static_cast<int>(slot_base), pl, n, pp,
                    static_cast<uint64_t>(timeout_s * 1e9), cur_stream());
}

// q [B, T, Hq, D], k/v [B, T, Hkv, D] bf16 contiguous -> (o [B, T, Hq, D], lse [B, Hq, T])
std::vector<Tensor> attention_fwd(Tensor q, Tensor k, Tensor v, double scale) {
  check_bf16_contig(q, "q");
  check_bf16_contig(k, "k");
  check_bf16_contig(v, "v");
  TORCH_CHECK(q.dim() == 4 && k.dim() == 4 && v.dim() == 4, "mmf: attention tensors are [B, T, H, D]");
  const c10::cuda::CUDAGuard guard(q.device());
  mmf::AttnArgs a{};
  a.B = static_cast<int>(q.size(0));
  a.T = static_cast<int>(q.size(1));
  a.Hq = static_cast<int>(q.size(2));
  a.D = static_cast<int>(q.size(3));
  a.Hkv = static_cast<int>(k.size(2));
  TORCH_CHECK(k.sizes() == v.sizes() && k.size(0) == a.B && k.size(1) == a.T && k.size(3) == a.D,
              "mmf: k/v shapes must match q");
  Tensor o = torch::empty_like(q);
  Tensor lse = torch::empty({a.B, a.Hq, a.T}, q.options().dtype(torch::kFloat32));
  a.q = q.data_ptr();
  a.k = k.data_ptr();
  a.v = v.data_ptr();
  a.o = o.data_ptr();
  a.lse = lse.data_ptr<float>();
  a.scale = static_cast<float>(scale);
  mmf::attention_fwd(a, cur_stream());
  return {o, lse};
}

std::vector<Tensor> attention_bwd(Tensor dout, Tensor q, Tensor k, Tensor v, Tensor o, Tensor lse, double scale) {
  check_bf16_contig(dout, "dout");
  check_bf16_contig(q, "q");
  check_bf16_contig(k, "k");
  check_bf16_contig(v, "v");
  check_bf16_contig(o, "o");
  TORCH_CHECK(lse.scalar_type() == torch::kFloat32 && lse.is_contiguous(), "mmf: lse must be contiguous fp32");
  const c10::cuda::CUDAGuard guard(q.device());
  mmf::AttnBwdArgs a{};
  a.B = static_cast<int>(q.size(0));
  a.T = static_cast<int>(q.size(1));
  a.Hq = static_cast<int>(q.size(2));
  a.D = static_cast<int>(q.size(3));
  a.Hkv = static_cast<int>(k.size(2));
  Tensor dq = torch::empty_like(q), dk = torch::empty_like(k), dv = torch::empty_like(v);
  Tensor delta = torch::empty({a.B, a.Hq, a.T}, q.options().dtype(torch::kFloat32));
  Tensor dk_h = torch::empty({a.B, a.T, a.Hq, a.D}, q.options().dtype(torch::kFloat32));
  Tensor dv_h = torch::empty({a.B, a.T, a.Hq, a.D}, q.options().dtype(torch::kFloat32));
  a.q = q.data_ptr();
  a.k = k.data_ptr();
  a.v = v.data_ptr();
  a.o = o.data_ptr();
  a.dout = dout.data_ptr();
  a.lse = lse.data_ptr<float>();
  a.delta = delta.data_ptr<float>();
  a.dk_h = dk_h.data_ptr<float>();
  a.dv_h = dv_h.data_ptr<float>();
  a.dq = dq.data_ptr();
  a.dk = dk.data_ptr();
  a.dv = dv.data_ptr();
  a.scale = static_cast<float>(scale);
  mmf::attention_bwd(a, cur_stream());
  return {dq, dk, dv};
}

int64_t device_error(int64_t device) {
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  return mmf::read_and_clear_device_error(static_cast<int>(device), cur_stream());
}

int64_t launch_count() { return static_cast<int64_t>(mmf::launch_count()); }

bool device_checks() {
#ifdef MMF_DEVICE_CHECKS
  return true;
#else
  return false;
#endif
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sm_100a kernels of my_muon_fsdp2_b200";
  m.def("ptr_table", &ptr_table);
  m.def("tc_gemm_ws", &tc_gemm_ws);
  m.def("tc_gemm_out", &tc_gemm_out);
  m.def("wgrad_out", &wgrad_out);
  m.def("ag_gemm", &ag_gemm);
  m.def("linear_gemm", &linear_gemm);
  m.def("wgrad_scatter", &wgrad_scatter);
  m.def("set_linear_split_tail", [](bool on) { mmf::set_linear_split_tail(on); });
  m.def("linear_resident_pairs", []() { return static_cast<int64_t>(mmf::linear_resident_pairs()); });
  m.def("rs_reduce", &rs_reduce);
  m.def("rs_pull_reduce", &rs_pull_reduce);
  m.def("muon_prep", &muon_prep);
  m.def("ns_scale", &ns_scale);
  m.def("ws_to_out", &ws_to_out);
  m.def("adamw", &adamw);
  m.def("muon_moments", &muon_moments);
  m.def("rmsnorm_fwd", &rmsnorm_fwd);
  m.def("rmsnorm_bwd", &rmsnorm_bwd);
  m.def("layernorm_fwd", &layernorm_fwd);
  m.def("embedding_fwd", &embedding_fwd);
  m.def("scale_", &scale_);
  m.def("clock_probe", [](Tensor out, int64_t cycles) {
    check_cuda(out, "out");
    TORCH_CHECK(out.scalar_type() == torch::kInt64 && out.is_contiguous() && out.dim() == 2 && out.size(1) == 2,
                "mmf: clock_probe writes an int64 [blocks, 2] tensor");
    const c10::cuda::CUDAGuard guard(out.device());
    mmf::clock_probe(cycles, static_cast<int>(out.size(0)), reinterpret_cast<long long*>(out.data_ptr<int64_t>()),
                     cur_stream());
  });
  m.def("embedding_bwd", &embedding_bwd);
  m.def("layernorm_bwd", &layernorm_bwd);
  m.def("rope_", &rope_);
  m.def("swiglu_fwd", &swiglu_fwd);
  m.def("swiglu_bwd", &swiglu_bwd);
  m.def("gelu_fwd", &gelu_fwd);
  m.def("gelu_bwd", &gelu_bwd);
  m.def("cross_entropy_", &cross_entropy_);
  m.def("power_iteration", &power_iteration);
  m.def("symm_barrier", &symm_barrier);
  m.def("attention_fwd", &attention_fwd);
  m.def("attention_bwd", &attention_bwd);
  m.def("set_attention_fwd_variant", [](int64_t v) { mmf::set_attention_fwd_variant(static_cast<int>(v)); });
  m.def("set_gemm_variant", [](int64_t v) { mmf::set_gemm_variant(static_cast<int>(v)); });
  m.def("gemm_variant", []() { return static_cast<int64_t>(mmf::gemm_variant()); });
  m.def("device_error", &device_error);
  m.def("launch_count", &launch_count);
  m.def("device_checks", &device_checks);
}
