// CUDA runtime behind the C ABI: loads a wire program (traced graph + plan
// metadata), plans storage and a launch list for it, and executes training
// steps / forward runs on one device stream, optionally inside a CUDA graph.
//
// This replaces the reference's WebGPU runtime (src/runtime.ts:157-499:
// one GPUBuffer per BufferSpec, one compute pass per IR op, writeback copies
// and a mapAsync per step) and its WGSL codegen (src/codegen.ts:48-56).
#pragma once
#include <cuda_runtime.h>
#include <cstdio>
#include <cstdlib>
#include <functional>
#include <map>
#include <set>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "json.hpp"
#include "kernels.cuh"

namespace tg {

// Error with a reference-style name ("Error", "ShapeError", "CudaError", ...).
struct TgError : std::runtime_error {
  std::string name;
  TgError(const std::string& n, const std::string& m) : std::runtime_error(m), name(n) {}
};

#define TG_CUDA(x)                                                                          \
  do {                                                                                      \
    cudaError_t e_ = (x);                                                                   \
    if (e_ != cudaSuccess)                                                                  \
      throw ::tg::TgError("CudaError", std::string(#x) + ": " + cudaGetErrorString(e_)); \
  } while (0)

struct TInfo {
  std::vector<int64_t> shape;
  int dtype = F32;
  int64_t numel = 1;
};

struct Writeback {
  int src;
  std::string dest;
  bool to_param;
};

// Parsed wire program. Field names mirror the reference's graph + BufferPlan
// vocabulary (src/ir.ts:284-296, src/buffers.ts:61-80).
// f32 of the decimal string x.toFixed(8): how the reference writes a float
// literal into its shader source (dropout p and scale).
inline float f32_lit8(double x) {
  char buf[64];
  snprintf(buf, sizeof buf, "%.8f", x);
  return (float)strtod(buf, nullptr);
}

// A kernel generated at plan time and compiled with NVRTC (jit.cu).
struct JitFn {
  std::string name, src;
  int device = 0;
  void* fn = nullptr;  // CUfunction, set by jit_compile_pending
};
std::shared_ptr<JitFn> jit_request(const std::string& name, const std::string& src);
void jit_compile_pending();
void jit_launch(const JitFn& f, unsigned grid_x, unsigned grid_y, unsigned block, void** args, cudaStream_t s);
const std::string& jit_preamble();

struct Program {
  tgjson::Value root;
  std::vector<TInfo> T;
  std::vector<const tgjson::Value*> ops;
  std::vector<std::string> kind;
  std::vector<int> out;
  std::vector<std::vector<int>> op_inputs;
  std::vector<int> producer;                 // tensor -> op index
  std::vector<std::vector<int>> consumers;   // tensor -> op indices (with repeats removed)
  std::vector<int> outputs;
  std::vector<std::pair<std::string, int>> captures;
  std::vector<std::pair<std::string, int>> params;  // graph order
  std::map<std::string, int> inputs;                // tensor_input name -> tensor
  struct State { std::string name; int tensor; double init; };
  std::vector<State> states;
  std::vector<std::pair<std::string, int>> grads;   // param name -> grad tensor
  std::vector<Writeback> writebacks;
  int loss = -1;
  int opt_start = -1;  // index of the first optimizer-pass op (= number of ops before it)
  const tgjson::Value* optimizer = nullptr;
  bool uses_prng = false;

  void parse(const char* json, size_t len);
  const tgjson::Value& op(int i) const { return *ops[i]; }
};

enum ArenaKind : int {
  AR_PARAM = 0, AR_GRAD, AR_M, AR_V, AR_STATE, AR_INPUT, AR_CONST, AR_PERSIST, AR_TEMP, AR_SCRATCH, AR_COUNT
};

// Where a tensor's elements live: a root tensor owns storage in an arena;
// views (reshape, stop_gradient, same-shape sum_to_shape/broadcast_to,
// leading-axis slices, permutes feeding GEMMs) point into their root with an
// element offset and strides. A virtual one-hot has no storage at all.
struct TView {
  int root = -1;
  int64_t off = 0;                 // element offset into the root's storage
  std::vector<int64_t> strides;    // element strides per dim
  bool contiguous = true;
  bool onehot = false;             // virtual one-hot of `onehot_idx` with depth shape.back()
  int onehot_idx = -1;
};

struct StorageLoc {
  int arena = -1;
  int64_t off = 0;  // bytes
  int64_t bytes = 0;
};

class Context;

// Elementwise op kinds, and an elementwise op's operand tensors in the order
// its expression reads them (runtime_fuse.cu).
const std::set<std::string>& ew_kinds();
std::vector<int> ew_operands(const Program& P, int i);

class Graph {
 public:
  Graph(Context* ctx, int id, Graph* parent, const char* json, size_t len);
  ~Graph();

  int id;
  Context* ctx;
  Graph* parent;
  Program P;

  // host API
  void upload_params(int n, const char* const* names, const float* const* data, const size_t* numel);
  void download_params(int n, const char* const* names, float* const* out, const size_t* numel);
  void set_inputs(int n, const char* const* names, const void* const* data, const size_t* bytes, bool device_src);
  void require_inputs(int n, const char* const* names) const;
  void launch_step();  // enqueue one step (scalars + kernels), no sync
  void read_loss(float* out);
  void read_output(void* out);
  void read_captures(void* const* out);
  void read_tensor(int t, void* out);
  void read_grad(const std::string& name, float* out);
  void reset_optimizer();
  void upload_states(int n, const char* const* names, const float* const* data, const size_t* numel);
  void download_states(int n, const char* const* names, float* const* out, const size_t* numel);
  int state_tensor(const std::string& name) const;
  // Per-step counters: optimizer steps taken and the PRNG seed counter.
  void get_counters(int64_t* step, int64_t* prng) const { *step = t_; *prng = prng_; }
  void set_counters(int64_t step, int64_t prng) { t_ = step; prng_ = prng; }
  void set_lr(const char* lr_json, size_t len);
  std::string info_json() const;
  float* param_ptr(const std::string& name) const;
  int64_t param_numel(const std::string& name) const;
  int launches_per_step() const { return (int)launches_.size(); }
  std::string launch_kinds() const;
  // Algorithmic bytes of each launch (each distinct tensor read once plus
  // every tensor written once), 0 where not accounted (GEMMs, collectives,
  // convolutions): the numerator of the memory-bound rooflines.
  const std::vector<double>& launch_bytes() const { return launch_bytes_; }
  const std::vector<std::string>& jit_sources() const { return jit_sources_; }
  // Runs one step launch by launch (no CUDA graph) with events around each
  // launch; fills per-launch milliseconds.
  void profile_step(std::vector<float>& ms);

 private:
  void plan();
  void plan_views();
  void plan_optimizer();
  void plan_storage();
  void plan_fusion();
  void emit_launches();
  // How an elementwise kernel of output shape oshape reads tensor t. Without
  // with_ptr (planning, before storage exists) only the mode is decided.
  EwInput ew_input(int t, const std::vector<int64_t>& oshape, bool& vec_ok, bool with_ptr = true);
  void emit_ew_group(int group, const int* seed_ptr, float* scratch, size_t scratch_floats,
                     const std::function<void(const std::string&, std::function<void(cudaStream_t)>)>& add);
  bool ew_internal(int t) const;
  bool ew_is_absorbed(int i) const { return !ew_absorbed_.empty() && ew_absorbed_[i]; }
  int ew_group_of(int i) const { return ew_group_.empty() ? -1 : ew_group_[i]; }
  void run_launches(cudaStream_t s);
  void init_constants();
  void* ptr(int t) const;
  const TView& view(int t) const { return views_[t]; }
  bool is_contig(int t) const { return views_[t].contiguous && !views_[t].onehot; }
  void host_scalars();

  std::vector<TView> views_;
  std::vector<int> action_;          // per op: planned action code
  std::vector<StorageLoc> loc_;      // per root tensor
  std::vector<int> op_done_;         // ops folded away
  std::vector<float> gemm_alpha_;    // per GEMM op: output scale folded in from a following mul_scalar
  // Fused causal attention blocks (plan_attention). Anchor ops carry action
  // 110 (forward: the PV GEMM) or 111 (backward: the first of its gradient
  // GEMMs, which writes dQ, dK, dV and dS); the other ops of a block are done.
  struct AttnBlock {
    int q, k, kt, v, o;            // forward tensors (k: the key view under the K^T permute)
    int dout, dv, ds, dq, dkt;     // backward tensors, -1 for a forward-only block
    int ml, rowdot;                // tensors whose storage holds (m, l) per row and rowsum(dO * O)
    int p_t;                       // the probabilities tensor (dropout index space)
    float scale, p, keep_scale;
    uint32_t salt;
    bool dropout;
  };
  std::vector<AttnBlock> attn_;
  std::map<int, int> attn_of_;                         // anchor op -> block
  std::map<int, std::pair<std::vector<int>, std::vector<int>>> fused_io_;  // op -> (reads, writes) for liveness
  std::map<int, int64_t> bytes_override_;              // root -> bytes, for holders smaller than their tensor
  std::map<int, int> softmax_drop_;                    // softmax_causal op -> dropout op it also evaluates
  std::set<std::pair<int, int>> no_read_;              // (op, tensor): the op's result is formed without reading it
  std::vector<int> eff_consumers(int t) const;         // consumers of t that read it
  std::map<int, std::vector<int>> extra_writes_;       // op -> further tensors its launch writes
  void plan_attention(const std::set<int>& observable);
  // Fused elementwise groups. A group is rooted at the op whose output it
  // writes: its last elementwise member, or a reduction that consumes it.
  struct EwGroup {
    std::vector<int> members;  // elementwise ops evaluated per element, ascending
    int root = -1;             // op whose output the launch writes
    int red = -1;              // the root when it is a reduction (sum_last, mean_last, sum_to_shape)
    // Row reductions only: groups of one value per row that read the
    // reduction's result, evaluated by the same kernel after the row sum
    // (their ops merged, ascending); each post root's output is written too.
    std::vector<int> post;
    std::vector<int> post_roots;
    // Row reductions only: a group over the reduction's input shape that reads
    // its per-row results, evaluated by the row's warp after them (ops
    // ascending); epi_root's output is written.
    std::vector<int> epi;
    int epi_root = -1;
    // Row reductions only: a plain row reduction (mean_last / sum_last of a
    // stored tensor over the same rows) computed by this launch as a first
    // pass over each row; its result is a register for the rest of the
    // kernel and is written too (LayerNorm's mean before its variance).
    int pre = -1;
    // Column reductions only: the elementwise group that produced the summed
    // tensor, whose value this launch also stores (its output has other
    // readers). The launch runs at that group's position.
    int wt = -1;
  };
  std::vector<EwGroup> ew_groups_;
  std::map<int, int> row_values(const EwGroup& G) const;
  bool reads_as_row(int x, const std::vector<int64_t>& vshape, int64_t len);
  std::set<int> wt_reds_;           // column reductions computed by their producer group's launch  // row value tensor -> the value it aliases
  std::vector<int> ew_group_;        // per op: group index when the op roots a group, else -1
  std::vector<char> ew_absorbed_;    // per op: value computed inside the groups that use it (no storage)
  std::vector<char> ew_post_;        // per op: absorbed as a row reduction's post op, output still stored
  bool jit_ = false;                 // fused elementwise groups compiled at plan time
  std::vector<std::string> jit_sources_;  // generated kernel sources (planning-only contexts)
  void* arena_[AR_COUNT] = {};
  int64_t arena_bytes_[AR_COUNT] = {};
  bool arena_owned_[AR_COUNT] = {};
  int64_t scratch_bytes_ = 0;
  std::map<std::string, int64_t> param_off_;   // byte offset in the param arena (or parent's)
  // Data parallel: each gradient written in place, with the index of the last
  // op before the optimizer section that touches it (its allreduce can start
  // after that op's launches); and the events that fork the gradient buckets
  // onto the communication stream and join them back.
  std::vector<std::pair<std::string, int>> grad_ready_;
  std::vector<cudaEvent_t> dp_events_;
  std::map<std::string, int64_t> param_n_;
  std::vector<std::pair<std::string, int>> layout_;  // flat arena order (name, numel)
  int64_t flat_floats_ = 0;  // padded total floats of the flat arenas
  int64_t n_decay_ = 0;
  // fused optimizer
  bool adam_fused_ = false, sgd_fused_ = false;
  AdamFlatDesc adam_{};
  SgdFlatDesc sgd_{};
  int adam_lrt_ = -1, adam_shrink_ = -1, sgd_lr_ = -1;
  // per-step host scalars
  int64_t t_ = 0;
  int64_t prng_ = 0;
  std::vector<std::function<void(cudaStream_t)>> launches_;
  std::vector<std::string> launch_kind_;
  std::vector<double> launch_bytes_;
  double next_bytes_ = 0;  // bytes of the next add()ed launch
  double tensor_bytes(int t) const;
  std::map<int, bool> causal_memo_;
  bool causal_zero(int t);  std::vector<std::function<void(cudaStream_t)>> post_;  // writebacks
  cudaGraph_t cgraph_ = nullptr;
  cudaGraphExec_t cexec_ = nullptr;
  bool use_graph_ = true;
  bool captured_ = false;
  float* loss_host_ = nullptr;  // pinned
  std::vector<std::pair<int, int64_t>> grad_copy_;  // (grad tensor, byte offset in the grad arena)
  int64_t loss_avg_off_ = 0;
  float scalar_host_[256] = {};  // pageable staging for per-step scalars
  int scalar_n_ = 0;
  tgjson::Value lr_override_;
  bool has_lr_override_ = false;
  friend class Context;
};

class Context {
 public:
  Context(int device, int rank, int world, const unsigned char* nccl_id);
  // Planning-only context: no device, stream or communicator. Graphs created
  // on it are planned in full (views, fusion, storage, launch list, generated
  // kernel sources) against placeholder arena addresses and never run.
  struct Dry {};
  Context(Dry, int world);
  ~Context();
  int device, rank, world;
  bool dry = false;
  cudaStream_t stream = nullptr;
  cudaStream_t comm_stream = nullptr;  // gradient allreduce buckets (world > 1)
  void* nccl = nullptr;  // ncclComm_t
  bool nccl_aborted = false;  // set after ncclCommAbort: every later step fails with NcclError
  int64_t dp_syncs = 0;       // completed data-parallel step waits (fault-injection counter)
  std::map<int, std::unique_ptr<Graph>> graphs;
  // Waits for the stream. With a communicator the wait polls: a CUDA error,
  // an asynchronous NCCL error, or no completion within TG_NCCL_TIMEOUT_S
  // aborts the communicator and throws NcclError, so a rank whose peer
  // stalled or left fails its step instead of hanging (the reference's
  // worker rejects every pending request when the worker dies).
  void sync(cudaStream_t s);
  void check_comm() const;  // throws NcclError once the communicator was aborted
  void allreduce_sum(float* buf, int64_t n, cudaStream_t s);
  // In-place sum allreduce of several ranges as one NCCL group.
  void allreduce_ranges(const std::vector<std::pair<float*, int64_t>>& ranges, cudaStream_t s);
};

}  // namespace tg
