// Host-side launch API of the native kernels.  Only plain C++/CUDA types cross this boundary,
// so the .cu translation units compile without the PyTorch headers; bindings.cpp adapts
// torch tensors to these calls.  Every launcher enqueues on the given stream and returns
// immediately; argument errors are thrown as std::runtime_error.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace mmf {

// ----------------------------------------------------------------------------------------
// Device error word shared by all kernels (bounded waits record their timeout code here).
int* device_error_word(int device);
int read_and_clear_device_error(int device, cudaStream_t stream);

// Number of kernel launches issued by this library since process start (host counter).
uint64_t launch_count();
void count_launch();

// ----------------------------------------------------------------------------------------
// tcgen05 GEMM:   V[b] = alpha_b * (A[b] @ Bop[b]) + beta_b * C[b]
//   A    : [batch, M, K] bf16 row-major (K contiguous)
//   Bop  : b_mn_major == false -> [batch, N, K] bf16 row-major (product uses Bop^T)
//          b_mn_major == true  -> [batch, K, N] bf16 row-major (product uses Bop as is)
//   C    : optional [batch, M, N] bf16 (may alias A when symmetric)
//   alpha_b = alpha * (alpha_vec ? alpha_vec[b] : 1), beta_b likewise.
// Requirements (checked): M % 128 == 0, N % 256 == 0, K % 64 == 0, 16-byte aligned bases.
//
// Epilogue "workspace" mode: D[b] = bf16(V[b]).  With symmetric == true (M == N and the
// product is symmetric, e.g. X X^T or A A for symmetric A) only tiles touching the upper
// triangle are computed and each upper element is also written to its mirror position.
struct GemmWsArgs {
  const void* A;
  const void* B;
  bool b_mn_major;
  void* D;
  const void* C;
  int batch, M, N, K;
  const float* alpha_vec;
  float alpha;
  const float* beta_vec;
  float beta;
  bool symmetric;
};
void tc_gemm_ws(const GemmWsArgs& args, cudaStream_t stream);

// GEMM kernel variant: 0 = automatic (CTA pair when the problem has enough 256-row tiles),
// 1 = single-CTA 128x256 tiles, 2 = CTA pair (cta_group::2) 256x256 tiles.
void set_gemm_variant(int v);
int gemm_variant();

// Epilogue "output" mode: for every element (i, j) with i < m_true, j < n_true, with
// (r, c) = transposed_b ? (j, i) : (i, j) the element's position in the destination matrix,
//   seg = r / seg_rows_b,  T = out_ptrs[b * nseg + seg],  idx = (r - seg * seg_rows_b) * ld_b + c
//   T[idx] = p_scale_b * T[idx] + v_scale_b * V[b][i][j]      (old value not read if p_scale_b == 0)
// Row segments let one launch scatter each rank's row shard into a different buffer (a local
// all-to-all staging segment or a peer's receive buffer).  Per-batch (ld, transposed,
// seg_rows) come from out_meta[3*b .. 3*b+2] when out_meta is non-null, else from the scalars.
struct GemmOutArgs {
  const void* A;
  const void* B;
  bool b_mn_major;
  bool a_mn_major;  // true: A is [batch, K, M] row-major (the product uses A^T); single-CTA kernel
  const void* C;
  int batch, M, N, K;
  const float* alpha_vec;
  float alpha;
  const float* beta_vec;
  float beta;
  const int64_t* out_ptrs;  // device array [batch * nseg]
  int nseg;
  const int64_t* out_meta;  // device array [batch * 3] or null
  int64_t out_ld;
  bool out_f32;
  bool out_transposed;
  int m_true, n_true;
  const float* p_scale_vec;  // device [batch] or null (-> p_scale)
  float p_scale;
  const float* v_scale_vec;  // device [batch] or null (-> v_scale)
  float v_scale;
};
void tc_gemm_out(const GemmOutArgs& args, cudaStream_t stream);

// ----------------------------------------------------------------------------------------
// Grouped GEMM of the transformer linears (linear_gemm.cu), CTA-pair tiles of 256 x 256:
//   out = epilogue(alpha * sum_k A[m, k] B[k, n])
// Operand storage (bf16, row-major, row pitch a multiple of 8 elements, 16-byte aligned):
//   a_mn == false: A segment s is [a_outer = rows, a_inner = K_s]          (K-major)
//   a_mn == true : A segment s is [a_outer = K,    a_inner = rows_s]       (the product uses A^T)
//   b_mn == false: B segment s is [b_outer = cols_s, b_inner = K]          (the product uses B^T)
//   b_mn == true : B segment s is [b_outer = K_s,  b_inner = cols]
// Supported pairs: (false, false) forward, (false, true) input gradient, (true, true) weight
// gradient.  Segments concatenate up to three operands along one axis:
//   LIN_SEG_M: A segments (rows seg_len[s]) -> out[s];  LIN_SEG_N: B segments (columns
//   seg_len[s]) -> out[s];  LIN_SEG_K: (A, B) pairs with reduction K[s], summed into out[0].
// Epilogues: see linear_gemm.cu.  Ragged M, N, K are handled (zero-filled loads, checked stores).
enum LinSegAxis : int { LIN_SEG_NONE = 0, LIN_SEG_M = 1, LIN_SEG_N = 2, LIN_SEG_K = 3 };
enum LinEpilogue : int {
  LIN_EPI_STORE = 0,
  LIN_EPI_ROPE = 1,
  LIN_EPI_SWIGLU = 2,
  LIN_EPI_SWIGLU_BWD = 3,
  LIN_EPI_GELU = 4,
  LIN_EPI_GELU_BWD = 5,
  LIN_EPI_SCATTER = 6,
};
struct LinearGemmArgs {
  int M, N;       // output rows and columns (SWIGLU: N = hidden units; LIN_SEG_M/N: the sum of seg_len)
  int K[3];       // reduction length (per segment for LIN_SEG_K, else K[0])
  bool a_mn, b_mn;
  int axis, nseg;
  int seg_len[3];
  const void* A[3];
  int64_t a_inner[3], a_outer[3];
  const void* B[3];
  int64_t b_inner[3], b_outer[3];
  int epilogue;
  void* out[3];   // STORE/ROPE: one per segment (or out[0]); SWIGLU: h, g, u; SWIGLU_BWD: dg, du; GELU: a, z
  int64_t ldo[3];
  bool out_f32, accumulate;
  float alpha;
  const void* C;  // STORE: + C (residual; may alias out[0]), pitch ldc
  int64_t ldc;
  const void* aux0;  // SWIGLU_BWD: g, GELU_BWD: z
  const void* aux1;  // SWIGLU_BWD: u
  int64_t ld_aux;
  const void* bias;  // STORE / GELU: + bias[col]
  int rope_mask;     // ROPE: bit s set -> rotate the heads of segment s
  int seq_len, head_dim;
  float rope_theta;
  // SCATTER (weight gradient, bf16): output row r goes to scatter_ptrs[r / scatter_rows] +
  // ((r % scatter_rows) * ldo[0] + col) elements (device table of nseg owner addresses, e.g. this
  // rank's sub-slot in every owner's receive buffer, peer-mapped); + C when given.
  const int64_t* scatter_ptrs;
  int scatter_nseg;
  int64_t scatter_rows;
};
void linear_gemm(const LinearGemmArgs& args, cudaStream_t stream);
// Split the tiles of a last, partly filled wave along K over the idle CTA pairs (default on).
void set_linear_split_tail(bool on);
// CTA pairs of the linear GEMM resident at once on the current device (its persistent grid).
int linear_resident_pairs();

// ----------------------------------------------------------------------------------------
// FSDP all-gather fused with the consuming GEMM:  Y[M, N] = X[M, K] @ W^T, where W [N, K] is
// row-sharded over `ws` ranks (rank s holds rows [s*N/ws, (s+1)*N/ws) at shard_ptrs[s], a
// peer-mapped address for s != rank).  The same launch assembles the full W into the local
// buffer G [N, K]: one extra warp per CTA pulls 128x64 pieces of the peers' shards (ring
// order starting at rank+1) with TMA loads and writes them into G with TMA stores, publishing
// a per-128-row-panel counter in `ready` [N/128] (zeroed by the launcher).  The GEMM visits
// its own shard's columns first, then the other shards in ring order, and reads a remote panel
// from G once it is complete; a panel that is not complete within `wait_ns` is read from the
// owner directly (never a wait without a bound, never a multicast load).
// Requirements: M % 128 == 0, K % 64 == 0, N % 256 == 0, (N / ws) % 128 == 0, ws <= 8.
struct AgGemmArgs {
  const void* X;
  int M, N, K;
  int rank, ws;
  int64_t shard_ptrs[8];
  void* G;
  void* Y;
  uint32_t* ready;
  uint64_t wait_ns;
};
void ag_gemm(const AgGemmArgs& args, cudaStream_t stream);

// Deterministic reduction of reduce-scatter slots: out[i] = bf16((accumulate ? out[i] : 0) +
// scale * sum_{s = 0..ws-1} slots[s * slot_stride + i]) with the sum taken in fp32 in rank order.
void rs_reduce(const void* slots, int ws, int64_t slot_stride, int64_t n, void* out, bool accumulate, float scale,
               cudaStream_t stream);

// Pull form of the same reduction: out[i] = bf16((accumulate ? out[i] : 0) + scale *
// sum_{s = 0..ws-1} srcs[s][offset + i]) where srcs (device array) holds every rank's partial
// buffer (peers through P2P mappings); fp32 sum in rank order.  n and offset multiples of 8.
void rs_pull_reduce(const int64_t* srcs, int ws, int64_t offset, int64_t n, void* out, bool accumulate, float scale,
                    cudaStream_t stream);

// ----------------------------------------------------------------------------------------
// Muon pre-NS multi-tensor kernel.  For matrix b (a row block of rows_b x cols_b elements):
//   mode 0 (copy):      u = g
//   mode 1 (ema):       buf = mu*buf + (1-mu)*g'            (lerp form)
//   mode 2 (heavy-ball):buf = mu*buf + g'
//   g' = g + wd_coupled * p  (only if wd_coupled != 0)
//   u = nesterov ? g' + mu*buf : buf   (modes 1, 2)
// then u is written as bf16 into dst_b at [dst_row0 + r][c] (or transposed [c][dst_row0 + r])
// with leading dimension dst_ld, and sum(u^2) is accumulated into sumsq[b] (fp32 atomics).
// If dst_b == 0 the update is applied directly: p = p_scale*p + v_scale*u (1-D params).
struct PrepDesc {
  int64_t grad;      // device pointer
  int64_t buf;       // fp32 momentum (0 in copy mode)
  int64_t param;     // param pointer (for coupled wd / direct apply), may be 0
  int64_t dst;       // bf16 destination base (0 -> direct apply)
  int32_t rows, cols;
  int32_t dst_row0;
  int32_t transposed;
  int64_t dst_ld;
  float p_scale, v_scale;  // direct-apply coefficients
};
struct PrepArgs {
  const PrepDesc* descs;  // device array [n]
  int n;
  int max_tiles;          // max over b of ceil(rows/64)*ceil(cols/64)
  int grad_f32;           // grad dtype: 0 bf16, 1 f32
  int param_f32;          // param dtype: 0 bf16, 1 f32
  int mode;
  int nesterov;
  float mu;
  float wd_coupled;
  float* sumsq;           // device [n] (may be null): += sum of squares of each tensor's update
  float* partials;        // device [n * muon_prep_blocks(max_tiles)] scratch when sumsq is set
  int vec8;               // all tensors allow 16-byte vector access (host-checked)
};
// Blocks per tensor of a muon_prep launch (the size of its per-block partial sums).
int muon_prep_blocks(int max_tiles);
// The sums of squares are reduced in a fixed order (per-block partials, then one warp per
// tensor), so the Frobenius scale and everything after it are bitwise reproducible.
void muon_prep(const PrepArgs& args, cudaStream_t stream);

// s[b] = 1 / (sqrt(sumsq[b]) + eps), s2[b] = s[b]^2 ; optionally sums `nparts` partials per
// matrix laid out as sumsq[p * n + b].
void ns_scale(const float* sumsq, int n, int nparts, float eps, float* s, float* s2, cudaStream_t stream);

// Elementwise copy of an (unscaled) bf16 workspace matrix to output pointers, applying
// T = p_scale*T + v_scale*s[b]*X (used when steps == 0 and for received NS results).
struct WsOutArgs {
  const void* X;  // [batch, Mp, Np] bf16 workspace
  int batch, Mp, Np;
  const float* s_vec;  // may be null
  const int64_t* out_ptrs;  // [batch * nseg]
  int nseg;
  const int64_t* out_meta;  // [batch * 3] (ld, transposed, seg_rows) or null
  int64_t out_ld;
  bool out_f32, out_transposed;
  int m_true, n_true;
  const float* p_scale_vec;
  float p_scale;
  const float* v_scale_vec;
  float v_scale;
};
void ws_to_out(const WsOutArgs& args, cudaStream_t stream);

// ----------------------------------------------------------------------------------------
// Multi-tensor AdamW (decoupled weight decay), fp32 moments, bf16 or fp32 params/grads.
struct AdamDesc {
  int64_t param, grad, exp_avg, exp_avg_sq;
  int64_t numel;
};
struct AdamArgs {
  const AdamDesc* descs;
  int n;
  int64_t max_numel;
  int param_f32, grad_f32;
  float lr, beta1, beta2, eps, weight_decay;
  float bias_correction1, bias_correction2_sqrt;  // host-computed
  int vec4;  // every tensor has numel % 4 == 0 and 16-byte aligned storage
};
void adamw_multi(const AdamArgs& args, cudaStream_t stream);

// State update of the reference update rule (reference muon_fsdp/fsdp.py:326-345), one pass per
// tensor: g = grad + wd p; buf = momentum buf + g; u = nesterov ? g + momentum buf : buf;
// sm = beta2 sm + (1 - beta2) u^2.  The descriptor fields map exp_avg -> momentum buffer and
// exp_avg_sq -> second moment (both fp32); the parameter is read, not written.
struct MomentArgs {
  const AdamDesc* descs;
  int n;
  int64_t max_numel;
  int param_f32, grad_f32;
  float momentum, beta2, weight_decay;
  int nesterov;
  int vec4;
};
void muon_moments_multi(const MomentArgs& args, cudaStream_t stream);

// ----------------------------------------------------------------------------------------
// Model kernels (bf16 activations, fp32 statistics).
void rmsnorm_fwd(const void* x, const void* w, void* y, float* rstd, int rows, int cols, float eps,
                 cudaStream_t stream);
void rmsnorm_bwd(const void* dy, const void* x, const void* w, const float* rstd, void* dx, float* dw_partial,
                 int rows, int cols, int partial_rows, cudaStream_t stream);
void layernorm_fwd(const void* x, const void* w, const void* b, void* y, float* mean, float* rstd, int rows,
                   int cols, float eps, cudaStream_t stream);
void layernorm_bwd(const void* dy, const void* x, const void* w, const float* mean, const float* rstd, void* dx,
                   float* dw_partial, float* db_partial, int rows, int cols, int partial_rows,
                   cudaStream_t stream);
void colsum_partials(const float* partial, int prow, int cols, void* out, bool out_f32, cudaStream_t stream);
// RoPE on x [tokens, heads, head_dim] (bf16, in place), positions = token % seq_len.
void rope_inplace(void* x, int tokens, int heads, int head_dim, int seq_len, float theta, bool inverse,
                  int64_t token_stride, int64_t head_stride, cudaStream_t stream);
void swiglu_fwd(const void* gate, const void* up, void* out, int64_t n, cudaStream_t stream);
void swiglu_bwd(const void* dout, const void* gate, const void* up, void* dgate, void* dup, int64_t n,
                cudaStream_t stream);
void gelu_fwd(const void* x, void* y, int64_t n, cudaStream_t stream);
void gelu_bwd(const void* dy, const void* x, void* dx, int64_t n, cudaStream_t stream);
// x (bf16, 16-byte aligned) *= s[0] (a device fp32 scalar).
// Diagnostic: `blocks` single-thread blocks each spin `cycles` SM cycles; out [blocks, 2] int64
// receives (cycles, nanoseconds) per block.
void clock_probe(int64_t cycles, int blocks, long long* out, cudaStream_t stream);
void scale_bf16(void* x, const float* s, int64_t n, cudaStream_t stream);
// Embedding rows (bf16, D % 8 == 0): out[t] = table[tokens[t]] (a token outside the table gives
// zeros and records ERR_BAD_ARGUMENT).  Backward: the dense table gradient in one pass from the
// sorted tokens and their permutation; `first` is int32 scratch of vocab entries.
void embedding_fwd(const void* table, const int64_t* tokens, void* out, int64_t n_tokens, int D, int64_t vocab,
                   cudaStream_t stream);
void embedding_bwd(const void* dy, const int64_t* sorted, const int64_t* perm, int* first, void* dtable,
                   int64_t n_tokens, int64_t vocab, int D, cudaStream_t stream);
// Softmax cross entropy over bf16 logits rows; writes per-row loss (fp32) and, when
// grad_scale != 0, overwrites logits with d(loss_sum*grad_scale)/dlogits (bf16).
void cross_entropy_fwd_bwd(void* logits, const int64_t* targets, float* loss_rows, int rows, int vocab,
                           int64_t ld, float grad_scale, int ignore_index, cudaStream_t stream);

// ----------------------------------------------------------------------------------------
// Spectral: batched power iteration helpers (GEMV with fused normalisation).
// work: max(m, n) + 1 floats; col_part: power_iteration_col_blocks(m) * n floats (the W^T u
// partial sums, added in a fixed order so that sigma is bitwise reproducible).
int power_iteration_col_blocks(int m);
void power_iteration(const void* W, bool w_f32, int m, int n, float* u, float* v, float* sigma, int iters,
                     float eps, float* work, float* col_part, cudaStream_t stream);

}  // namespace mmf
