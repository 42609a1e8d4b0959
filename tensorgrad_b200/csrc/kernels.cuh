// Kernel-side data structures and host launch wrappers shared by the planner.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>
#include <cstddef>
#include <functional>
#include <string>

namespace tg {

enum DType : int { F32 = 0, I32 = 1, BOOL = 2 };

int device_sm_count();

// ---------------------------------------------------------------------------
// Elementwise program ("EW"): one kernel evaluates a straight-line program of
// elementwise IR ops over every element of a common output shape. Inputs are
// read through broadcast index maps; several program values can be stored.
// A single op is a one-instruction program; the fusion pass merges chains of
// same-shape elementwise ops into one program so intermediates stay in
// registers instead of round-tripping HBM.
// ---------------------------------------------------------------------------
constexpr int EW_MAX_IN = 8;
constexpr int EW_MAX_OUT = 4;
constexpr int EW_MAX_INSTR = 40;
constexpr int EW_MAX_RANK = 6;
constexpr int EW_NREG = 8;

enum EwInMode : int {
  IN_FULL = 0,     // same shape as output, contiguous: offset = i
  IN_SCALAR = 1,   // one element: offset = 0
  IN_PERIOD = 2,   // trailing-suffix broadcast: offset = i % period
  IN_ROWDIV = 3,   // leading-prefix broadcast ([..., 1] over [..., D]): offset = i / period
  IN_STRIDED = 4,  // general: offset = sum(coord_d * stride_d)
  IN_ONEHOT = 5,   // virtual one-hot of int indices at ptr: (idx[i/period] == i%period) ? 1 : 0
};

struct EwInput {
  const void* ptr;
  int mode;
  int dtype;
  int64_t period;
  int64_t strides[EW_MAX_RANK];
};

enum EwOp : uint8_t {
  EW_LOAD = 0,  // dst <- input[a]
  EW_ADD, EW_SUB, EW_MUL, EW_DIV, EW_MIN, EW_MAX,
  EW_MULS, EW_ADDS,  // dst <- a (*|+) imm
  EW_SQRT, EW_RSQRT, EW_LOG, EW_EXP, EW_RELU, EW_NEG, EW_ABS, EW_TANH, EW_SIGMOID, EW_ERF,
  EW_SIN, EW_COS,
  EW_LESS, EW_GREATER,    // dst <- (a op b) ? 1 : 0 as int bits (aux=1: compare as i32)
  EW_WHERE,               // dst <- a(int bits) != 0 ? b : c   (bits preserved)
  EW_RELU_GRAD,           // dst <- a > 0 ? b : 0
  EW_DROPOUT,             // dst <- a * mask(seed, salt=aux, i); imm = f32(p), imm2 = f32(scale)
  EW_WHERE_CAUSAL,        // dst <- (k <= q) ? a : imm ; aux = T
  EW_ADAM_M,              // dst <- imm*a + imm2*b
  EW_ADAM_V,              // dst <- imm*a + imm2*b*b
  EW_ADAM_P,              // dst <- d*a - (c*b)/(sqrt(e)+imm)  a=p b=m c=lrt d=shrink e=v
  EW_COPY,                // dst <- a
  EW_CONST,               // dst <- imm (bits from aux when c==1)
};

struct EwInstr {
  uint8_t op, dst, a, b, c, d, e, pad;
  float imm, imm2;
  uint32_t aux;
};

struct EwProgram {
  int64_t numel;
  int rank;
  int n_in, n_out, n_instr;
  int64_t dims[EW_MAX_RANK];
  EwInput in[EW_MAX_IN];
  void* out[EW_MAX_OUT];
  uint8_t out_reg[EW_MAX_OUT];
  const int* seed;      // __prngSeed device scalar (dropout)
  int64_t drop_offset;  // global element offset of this shard (data parallel)
  int vec4;             // all inputs/outputs allow 4-wide access
  EwInstr code[EW_MAX_INSTR];
};

void launch_ew(const EwProgram& p, cudaStream_t s);

// ---------------------------------------------------------------------------
// Row kernels: reductions and softmaxes along the last axis.
// ---------------------------------------------------------------------------
enum RowKind : int { ROW_SUM = 0, ROW_MEAN, ROW_ARGMAX, ROW_LOGSOFTMAX, ROW_SOFTMAX_CAUSAL, ROW_CATEGORICAL };
// x: [rows, D] contiguous. For ROW_SUM/MEAN/ARGMAX/CATEGORICAL out has `rows`
// elements; for softmaxes out is [rows, D]. For softmax_causal, row r is
// query position r % D.
void launch_row(int kind, const float* x, void* out, int64_t rows, int64_t D, cudaStream_t s,
                const int* seed = nullptr, uint32_t salt = 0, float* scratch = nullptr,
                size_t scratch_floats = 0);
// softmax_causal rows of D <= 1024 that also write dropout(softmax) to out2:
// element e of the [rows, D] result keeps when the hash of
// (seed ^ salt ^ (u32)(drop_off + e)) / 2^32 >= p and is scaled by keep_scale,
// exactly as the elementwise dropout kernels decide. Returns false (nothing
// launched) for rows too long for the register path.
struct RowDropout {
  float* out2;
  const int* seed;
  uint32_t salt;
  float p, keep_scale;
  int64_t drop_off;
};
bool launch_softmax_causal_dropout(const float* x, float* out, int64_t rows, int64_t D, const RowDropout& d,
                                   cudaStream_t s);
// Scratch floats launch_row uses (long-row split path); 0 when none.
size_t row_scratch_floats(int kind, int64_t rows, int64_t D);

// Column sums [outer, inner] -> [inner] (deterministic two-pass with scratch).
size_t colsum_scratch_floats(int64_t outer, int64_t inner);
// Chunking of the two-pass column sum (chunks of consecutive rows) and its
// second pass, shared with generated kernels that compute the first pass.
int64_t colsum_chunks(int64_t outer, int64_t inner);
int64_t colsum_col_blocks(int64_t inner, bool vec);
void launch_colsum_fold(const float* part, float* out, int64_t nchunk, int64_t inner, cudaStream_t s);
void launch_colsum(const float* x, float* out, int64_t outer, int64_t inner, float* scratch, cudaStream_t s);
// General sum-to-shape: keep[d] = 1 where the output keeps input axis d.
// out[c] = sum of x[b, c, i] over b < R1, i < R2 (deterministic two-pass).
int64_t sum_mid_scratch_floats(int64_t R1, int64_t K);
void launch_sum_mid(const float* x, float* out, int64_t R1, int64_t K, int64_t R2, float* scratch, cudaStream_t s);
void launch_sum_general(const float* x, float* out, int rank, const int64_t* in_dims, const int64_t* keep,
                        int64_t in_numel, int64_t out_numel, cudaStream_t s);

// ---------------------------------------------------------------------------
// Strided copy: out[sum c*out_strides] = in[sum c*in_strides] over dims.
// Covers permute, slice_range, concat pieces, scatter_axis, broadcast copies.
// ---------------------------------------------------------------------------
constexpr int CP_MAX_RANK = 8;
struct CopyDesc {
  int rank;
  int64_t dims[CP_MAX_RANK];
  int64_t in_strides[CP_MAX_RANK];
  int64_t out_strides[CP_MAX_RANK];
  int64_t numel;
};
void launch_copy(const CopyDesc& d, const void* in, void* out, cudaStream_t s);
// Fused causal attention (kernels_attn.cu). A view addresses element
// (b, h, t, c) at p[b*s0 + h*s1 + t*s2 + c*s3].
struct AttnView { float* p; int64_t s0, s1, s2, s3; };
struct AttnParams {
  int B, H, T, D;
  AttnView q, k, v, o, dout, dq, dk, dv;
  float* ml;       // [B*H*T][2]: each query row's max and sum (forward writes, backward reads)
  float* dv_row;   // [B*H*T]: rowsum(dO * O)
  float* ds;       // dS rows [B*H*T][ds_ld]; only blocks on or below the diagonal are written
  int64_t ds_ld;
  float scale, p, keep_scale;
  uint32_t salt;   // dropout salt, already mixed as the elementwise dropout mixes it
  int dropout;
  const int* seed;
  int64_t drop_off;
};
bool attn_supported_dim(int d);
void launch_attn_fwd(const AttnParams& P, cudaStream_t s);
// tcgen05 forward (head dim 64, no dropout, unit head-dim stride; opt-in with
// TG_ATTN_TC=1); false when the block is not taken (the warp-MMA forward runs
// instead).
bool launch_attn_fwd_tc(const AttnParams& P, cudaStream_t s);
int attn_tc_error_flag(bool reset);
void launch_attn_bwd(const AttnParams& P, cudaStream_t s);
// Row-strided copy to a new row stride (operand staging for TMA).
void launch_pad_rows(const float* src, int64_t ld_src, float* dst, int64_t ld_dst, int64_t rows, int64_t cols,
                     cudaStream_t s);
void launch_fill(void* out, int64_t n, uint32_t bits, cudaStream_t s);
// One thread that waits ns nanoseconds of GPU time (%globaltimer) and exits:
// holds the stream while the host enqueues a profiled step behind it.
void launch_gpu_delay(uint64_t ns, cudaStream_t s);
void launch_arange(void* out, int64_t n, int dtype, cudaStream_t s);
void launch_one_hot(const int* idx, void* out, int64_t n_idx, int64_t depth, int dtype, cudaStream_t s);
void launch_randn(float* out, int64_t n, const int* seed, uint32_t salt_const, cudaStream_t s);

// ---------------------------------------------------------------------------
// GEMM: C[b] (+)= alpha * A[b] @ B[b] (+ bias) with arbitrary strides.
// ---------------------------------------------------------------------------
struct GemmDesc {
  int64_t M, N, K, batch;  // batch index z = i1 * batch2 + i2, i1 < batch / batch2
  const float* A; int64_t lda_m, lda_k, a_batch;  // A(m,k) = A[m*lda_m + k*lda_k]
  const float* B; int64_t ldb_k, ldb_n, b_batch;  // B(k,n) = B[k*ldb_k + n*ldb_n]
  float* C; int64_t ldc, c_batch;                 // C(m,n) = C[m*ldc + n*ldc_n]
  const float* bias;                              // optional [N], added in the epilogue
  float alpha;
  int accumulate;                                 // C += result
  int64_t batch2;                                 // inner batch extent (1 = single batch dim)
  int64_t a_batch2, b_batch2, c_batch2;           // strides of the inner batch index
  int64_t ldc_n;                                  // C column stride (0 is read as 1)
  // Causal structure of A (square M == K, batched attention): 1 = A(m, k) is
  // exactly zero for k > m (a causal softmax, or a product with one), so the
  // rows of a tile need only k below the tile's end; 2 = zero for k < m (the
  // transpose), the rows need only k from the tile's start. 0 = dense.
  // tri_cols: the same for B's columns (B(k, n) zero for k > n: 1; k < n: 2).
  int tri;
  int tri_cols;
  float* workspace;                               // split-K partial tiles (may be null)
  int64_t workspace_floats;
};
// K-splits the tensor-core GEMM would use for this problem (1 = none) and the
// workspace floats that needs.
int gemm_tc_splits(int64_t M, int64_t N, int64_t K, int64_t batch);
int64_t gemm_tc_workspace_floats(int64_t M, int64_t N, int64_t K, int64_t batch);
void launch_gemm_simt(const GemmDesc& g, cudaStream_t s);
// tcgen05/TMEM 3xTF32 GEMM; returns false when the shape/layout is not taken.
bool launch_gemm_tc(const GemmDesc& g, cudaStream_t s);
// Error code a tcgen05 GEMM recorded after a bounded wait ran out (0 = none).
int gemm_tc_error_flag(bool reset);
int gemm_tc_debug(int* out8);
int gemm_tc_trace(long long* out, int cap);

// Embedding gather: out[r, :] = table[idx[r], :] (0 where idx out of range).
void launch_gather_rows(const int* idx, const float* table, float* out, int64_t rows, int64_t V,
                        int64_t D, cudaStream_t s);
// Deterministic embedding backward: dtable[v,:] = sum of dy[r,:] over rows r
// with idx[r]==v, in ascending r (stable counting sort, no float atomics).
size_t embedding_grad_scratch_ints(int64_t rows, int64_t V, int64_t D);
void launch_embedding_grad(const int* idx, const float* dy, float* dtable, int64_t rows, int64_t V,
                           int64_t D, int* scratch, cudaStream_t s);
// out[r] = g[r] where 0 <= t[r] < V, else 0 (the row sum of g[r] * oneHot(t)[r])
void launch_row_hit(const float* g, const int* t, float* out, int64_t rows, int64_t V, cudaStream_t s);
// Row pick: out[r] = x[r, t[r]] (0 if out of range)
void launch_pick(const float* x, const int* t, float* out, int64_t rows, int64_t V, cudaStream_t s);

// ---------------------------------------------------------------------------
// conv2d / pool (NCHW)
// ---------------------------------------------------------------------------
struct ConvDesc {
  int B, Cin, H, W, Cout, kH, kW, Hout, Wout, sH, sW, pH, pW, G;
};
// conv2d and both gradients as column gathers plus GEMMs (kernels_conv.cu).
// `which`: 0 forward (in0 = x, in1 = w, out = y), 1 input grad (w, dy, dx),
// 2 weight grad (x, dy, dw). emit_conv hands each launch, labelled, to `add`.
using ConvEmit = std::function<void(const std::string&, std::function<void(cudaStream_t)>)>;
int64_t conv_gemm_scratch_floats(const ConvDesc& c, int which);
void emit_conv(int which, const ConvDesc& c, const float* in0, const float* in1, float* out, float* scratch,
               int64_t scratch_floats, const ConvEmit& add);
void launch_maxpool(const ConvDesc& c, const float* x, float* y, cudaStream_t s);
void launch_maxpool_grad(const ConvDesc& c, const float* x, const float* dy, float* dx, cudaStream_t s);

// ---------------------------------------------------------------------------
// Fused multi-tensor Adam/AdamW over flat arenas (in place).
// Elements [0, n_decay) use `shrink` (device scalar or literal); the rest 1.
// ---------------------------------------------------------------------------
struct AdamFlatDesc {
  float* p; float* m; float* v; const float* g;
  int64_t n, n_decay;
  float beta1, one_minus_beta1, beta2, one_minus_beta2, eps;
  const float* lrt;           // device scalar
  const float* shrink_dev;    // device scalar or nullptr
  float shrink_lit;
  float grad_scale;           // multiplies g (1/world for data-parallel averaging)
};
void launch_adam_flat(const AdamFlatDesc& d, cudaStream_t s);

// SGD over flat arenas (in place): g_eff = g*scale (+wd*p for decayed);
// v = mu*v + g_eff; upd = nesterov ? g_eff + mu*v : v; p -= lr*upd.
struct SgdFlatDesc {
  float* p; float* v; const float* g;
  int64_t n, n_decay;
  float momentum, wd;
  int nesterov;
  const float* lr;
  float grad_scale;
};
void launch_sgd_flat(const SgdFlatDesc& d, cudaStream_t s);

// Scale a flat buffer in place (data-parallel gradient averaging).
void launch_scale(float* x, int64_t n, float s, cudaStream_t st);

}  // namespace tg
