// Planner part 2 (storage, launch list) and execution.
#include <nccl.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <atomic>
#include <chrono>
#include <memory>
#include <set>
#include <thread>

#include "runtime.hpp"

namespace tg {

static std::vector<int64_t> cstrides(const std::vector<int64_t>& shape) {
  std::vector<int64_t> s(shape.size(), 1);
  for (int i = (int)shape.size() - 2; i >= 0; --i) s[i] = s[i + 1] * shape[i + 1];
  return s;
}
static int64_t align256(int64_t b) { return (b + 255) / 256 * 256; }
static bool is_leaf_kind(const std::string& k) {
  return k == "param_input" || k == "tensor_input" || k == "state_input";
}
static bool is_const_kind(const std::string& k) {
  return k == "const_scalar" || k == "const_fill" || k == "arange";
}

// Learning-rate schedule at a 1-based step (restates src/lr.ts:69-101).
static double resolve_lr(const tgjson::Value& s, int64_t step) {
  if (s.kind == tgjson::Value::Num) return s.n;
  const std::string& k = s["kind"].str();
  int64_t start = 0;
  if (auto* ss = s.find("startStep")) if (!ss->is_null()) start = ss->i64();
  int64_t st = std::max<int64_t>(1, step - start);
  if (k == "linear") {
    double f = std::min(1.0, (double)st / s["steps"].num());
    return s["peak"].num() + (s["final"].num() - s["peak"].num()) * f;
  }
  if (k == "cosineAnnealing") {
    double f = std::min(1.0, (double)st / s["steps"].num());
    return s["final"].num() + 0.5 * (s["peak"].num() - s["final"].num()) * (1 + std::cos(M_PI * f));
  }
  if (k == "warmup") {
    if (st <= s["steps"].i64()) return s["peak"].num() * ((double)st / s["steps"].num());
    return resolve_lr(s["after"], st - s["steps"].i64());
  }
  if (k == "staircase") return s["peak"].num() * std::pow(s["gamma"].num(), (double)((st - 1) / s["every"].i64()));
  if (k == "multiStep") {
    int n = 0;
    for (auto& m : s["milestones"].a) if (st >= m.i64()) ++n;
    return s["peak"].num() * std::pow(s["gamma"].num(), (double)n);
  }
  throw TgError("Error", "unknown lr schedule kind " + k);
}

// ------------------------------------------------------------------ Graph --
Graph::Graph(Context* c, int gid, Graph* par, const char* json, size_t len) : id(gid), ctx(c), parent(par) {
  P.parse(json, len);
  const char* ng = getenv("TG_NO_GRAPH");
  use_graph_ = !(ng && ng[0] == '1');
  if (!ctx->dry) TG_CUDA(cudaMallocHost(&loss_host_, 64));
  plan();
}

Graph::~Graph() {
  for (auto e : dp_events_) cudaEventDestroy(e);
  // A captured step of an aborted communicator keeps NCCL resources that the
  // abort already released: it is left to process exit rather than destroyed.
  const bool keep = ctx && ctx->nccl_aborted;
  if (cexec_ && !keep) cudaGraphExecDestroy(cexec_);
  if (cgraph_ && !keep) cudaGraphDestroy(cgraph_);
  for (int a = 0; a < AR_COUNT; ++a)
    if (arena_owned_[a] && arena_[a]) cudaFree(arena_[a]);
  if (loss_host_) cudaFreeHost(loss_host_);
}

void Graph::plan() {
  action_.assign(P.ops.size(), 0);
  op_done_.assign(P.ops.size(), 0);
  gemm_alpha_.assign(P.ops.size(), 1.f);
  for (size_t i = 0; i < P.ops.size(); ++i) {
    if (is_leaf_kind(P.kind[i]) || is_const_kind(P.kind[i])) op_done_[i] = 1;
  }
  plan_views();
  plan_optimizer();
  if (ctx->world > 1 && !parent && P.optimizer && !adam_fused_ && !sgd_fused_)
    throw TgError("Error", "data-parallel training needs the fused optimizer path; this optimizer graph "
                           "does not match the Adam/AdamW/SGD update patterns");
  plan_fusion();
  plan_storage();
  if (!ctx->dry) init_constants();
  emit_launches();
}

void* Graph::ptr(int t) const {
  const TView& v = views_[t];
  if (v.onehot) return nullptr;
  int r = v.root;
  const StorageLoc& L = loc_[r];
  if (L.arena < 0) throw TgError("Error", "internal: tensor #" + std::to_string(t) + " has no storage");
  char* base = reinterpret_cast<char*>(arena_[L.arena]);
  return base + L.off + v.off * 4;
}

float* Graph::param_ptr(const std::string& name) const {
  const Graph* g = this;
  while (g->parent) g = g->parent;
  auto it = g->param_off_.find(name);
  if (it == g->param_off_.end()) return nullptr;
  return reinterpret_cast<float*>(reinterpret_cast<char*>(g->arena_[AR_PARAM]) + it->second);
}
int64_t Graph::param_numel(const std::string& name) const {
  const Graph* g = this;
  while (g->parent) g = g->parent;
  auto it = g->param_n_.find(name);
  return it == g->param_n_.end() ? -1 : it->second;
}

// Scratch bytes an op's launch needs (shared buffer: launches are serial).
// Whether the kept dims of a reduction form one contiguous run with reduced
// dims on both sides ([R1, K, R2] after merging); fills the three extents.
static bool mid_runs(const std::vector<int64_t>& is, const std::vector<int64_t>& keep, int64_t* r3) {
  int64_t e[3] = {1, 1, 1};
  int phase = 0;  // 0: leading reduced, 1: kept, 2: trailing reduced
  for (size_t d = 0; d < is.size(); ++d) {
    if (is[d] == 1) continue;
    if (keep[d]) {
      if (phase == 2) return false;
      phase = 1;
    } else if (phase == 1) {
      phase = 2;
    }
    e[phase] *= is[d];
  }
  if (phase != 2 || e[0] == 1) return false;
  if (r3) { r3[0] = e[0]; r3[1] = e[1]; r3[2] = e[2]; }
  return true;
}

static int64_t scratch_for(const Program& P, int i, int action) {
  const std::string& k = P.kind[i];
  if (action == 101) {
    int b = P.op(i)["b"].i32();
    int a = P.op(i)["a"].i32();  // permute([K=V, rows])
    int64_t V = P.T[a].shape[0];
    int64_t rows = P.T[b].shape[0];
    return (int64_t)embedding_grad_scratch_ints(rows, V, P.T[b].shape[1]) * 4;
  }
  if (k == "sum_last" || k == "mean_last") {
    int a = P.op(i)["a"].i32();
    int64_t D = P.T[a].shape.back();
    return (int64_t)row_scratch_floats(k == "sum_last" ? ROW_SUM : ROW_MEAN, P.T[a].numel / std::max<int64_t>(D, 1), D) * 4;
  }
  if (k == "matmul" || k == "matmul_batched") {
    const auto& os = P.T[P.out[i]].shape;
    int a = P.op(i)["a"].i32();
    int64_t K = P.T[a].shape.back(), N = os.back(), M = os[os.size() - 2], batch = 1;
    for (size_t d = 0; d + 2 < os.size(); ++d) batch *= os[d];
    // either the batch folds into M (matmul) or stays a batch: same M*N*batch
    int64_t f = std::max(gemm_tc_workspace_floats(M * batch, N, K, 1), gemm_tc_workspace_floats(M, N, K, batch));
    // room to copy both operands to 16-byte row strides (see the GEMM emission)
    if (M % 4 || N % 4 || K % 4) {
      auto up4 = [](int64_t v) { return (v + 3) / 4 * 4; };
      const int64_t m = M * batch;
      f = (f + 63) / 64 * 64 + std::max(m * up4(K), K * up4(m)) + std::max(N * up4(K), K * up4(N)) + 128;
    }
    return 4 * f;
  }
  if (k == "conv2d" || k == "conv2d_input_grad" || k == "conv2d_weight_grad") {
    const auto& O = P.op(i);
    const auto& os = P.T[P.out[i]].shape;
    ConvDesc c{};
    c.sH = O["strideH"].i32(); c.sW = O["strideW"].i32(); c.pH = O["padH"].i32(); c.pW = O["padW"].i32();
    c.G = O.find("groups") ? O["groups"].i32() : 1;
    int which = 0;
    if (k == "conv2d") {
      auto& xs = P.T[O["input"].i32()].shape; auto& ws = P.T[O["weight"].i32()].shape;
      c.B = (int)xs[0]; c.Cin = (int)xs[1]; c.H = (int)xs[2]; c.W = (int)xs[3];
      c.Cout = (int)ws[0]; c.kH = (int)ws[2]; c.kW = (int)ws[3]; c.Hout = (int)os[2]; c.Wout = (int)os[3];
    } else if (k == "conv2d_input_grad") {
      auto& ws = P.T[O["weight"].i32()].shape; auto& ds = P.T[O["dy"].i32()].shape;
      c.B = (int)os[0]; c.Cin = (int)os[1]; c.H = (int)os[2]; c.W = (int)os[3];
      c.Cout = (int)ws[0]; c.kH = (int)ws[2]; c.kW = (int)ws[3]; c.Hout = (int)ds[2]; c.Wout = (int)ds[3];
      which = 1;
    } else {
      auto& xs = P.T[O["input"].i32()].shape; auto& ds = P.T[O["dy"].i32()].shape;
      c.B = (int)xs[0]; c.Cin = (int)xs[1]; c.H = (int)xs[2]; c.W = (int)xs[3];
      c.Cout = (int)os[0]; c.kH = (int)os[2]; c.kW = (int)os[3]; c.Hout = (int)ds[2]; c.Wout = (int)ds[3];
      which = 2;
    }
    return conv_gemm_scratch_floats(c, which) * 4;
  }
  if (k == "sum_to_shape") {
    int a = P.op(i)["a"].i32();
    int64_t inner = P.T[P.out[i]].numel, outer = P.T[a].numel / std::max<int64_t>(inner, 1);
    int64_t f = std::max<int64_t>(colsum_scratch_floats(outer, inner), row_scratch_floats(ROW_SUM, inner, outer));
    return std::max<int64_t>(f, sum_mid_scratch_floats(outer, inner)) * 4;
  }
  return 0;
}

void Graph::plan_storage() {
  const int nT = (int)P.T.size(), nO = (int)P.ops.size();
  loc_.assign(nT, StorageLoc{});
  std::vector<int> cls(nT, -1);
  std::set<int> pinned;
  for (int t : P.outputs) pinned.insert(views_[t].root);
  for (auto& c : P.captures) pinned.insert(views_[c.second].root);
  for (auto& w : P.writebacks) pinned.insert(views_[w.src].root);

  // Which roots are read or written by remaining launches.
  std::vector<int> used(nT, 0), def(nT, -1), end(nT, -1);
  // end[] restricted to ops before the optimizer section (gradient readiness)
  std::vector<int> end_bwd(nT, -1);
  const int opt_stop = P.opt_start >= 0 ? P.opt_start : nO;
  auto bump_end = [&](int r, int i) {
    end[r] = std::max(end[r], i);
    if (i < opt_stop) end_bwd[r] = std::max(end_bwd[r], i);
  };
  auto touch = [&](int t, int i) {
    const TView& v = views_[t];
    int r = v.onehot ? views_[v.onehot_idx].root : v.root;
    used[r] = 1;
    bump_end(r, i);
  };
  for (int i = 0; i < nO; ++i) {
    if (op_done_[i]) continue;
    // An absorbed elementwise op has no output; the groups that evaluate it
    // read its operands at their own positions.
    if (ew_is_absorbed(i)) continue;
    auto fio = fused_io_.find(i);
    if (fio != fused_io_.end()) {  // a fused block: its own read and write sets
      for (int w : fio->second.second) {
        const int r = views_[w].root;
        used[r] = 1;
        if (def[r] < 0 || i < def[r]) def[r] = i;
        bump_end(r, i);
      }
      for (int t : fio->second.first) touch(t, i);
      continue;
    }
    int o = P.out[i];
    // The op writes its output's root: its own storage, or (for a GEMM or
    // permute writing straight into a later permute's layout) that root.
    if (!views_[o].onehot) {
      const int r = views_[o].root;
      used[r] = 1;
      if (def[r] < 0 || i < def[r]) def[r] = i;
      bump_end(r, i);
    }
    if (action_[i] == 103) {  // row hit: reads g and the one-hot's indices
      const int m = P.producer[P.op(i)["a"].i32()];
      for (const char* f : {"a", "b"}) {
        const int t = P.op(m)[f].i32();
        touch(views_[t].onehot ? P.op(P.producer[t])["indices"].i32() : P.op(P.producer[t])["a"].i32(), i);
      }
      int o = P.out[i];
      const int r = views_[o].root;
      used[r] = 1;
      if (def[r] < 0 || i < def[r]) def[r] = i;
      bump_end(r, i);
      continue;
    }
    if (action_[i] == 102) {  // pick: reads x and the one-hot's indices
      const int m = P.producer[P.op(i)["a"].i32()];
      for (const char* f : {"a", "b"}) {
        const int t = P.op(m)[f].i32();
        touch(views_[t].onehot ? P.op(P.producer[t])["indices"].i32() : t, i);
      }
      continue;
    }
    if (action_[i] == 100 || action_[i] == 101) {
      int a = P.op(i)["a"].i32();
      int oh = action_[i] == 100 ? a : P.op(P.producer[P.op(P.producer[a])["a"].i32()])["a"].i32();
      int idx = P.op(P.producer[oh])["indices"].i32();
      touch(idx, i);
      touch(P.op(i)["b"].i32(), i);
      continue;
    }
    const int g = ew_group_of(i);
    if (g >= 0) {
      for (int m : ew_groups_[g].members)
        for (int t : P.op_inputs[m])
          if (!ew_internal(t)) touch(t, i);
      const EwGroup& G = ew_groups_[g];
      for (int pr : G.post_roots) {  // the kernel also writes the post ops' results
        const int r = views_[P.out[pr]].root;
        used[r] = 1;
        if (def[r] < 0 || i < def[r]) def[r] = i;
        bump_end(r, i);
      }
      if (G.pre >= 0) touch(P.op(G.pre)["a"].i32(), i);  // the absorbed first-pass reduction's input
      if (G.epi_root >= 0) {  // and the epilogue group's result
        const int r = views_[P.out[G.epi_root]].root;
        used[r] = 1;
        if (def[r] < 0 || i < def[r]) def[r] = i;
        bump_end(r, i);
        for (int m : G.epi)
          for (int t : P.op_inputs[m])
            if (!ew_internal(t)) touch(t, i);
      }
      if (!G.post_roots.empty()) {
        for (int m : G.post)
          for (int t : P.op_inputs[m])
            if (!ew_internal(t)) touch(t, i);
      }
    }
    for (int t : P.op_inputs[i])
      if (!ew_internal(t)) touch(t, i);
    auto xw = extra_writes_.find(i);
    if (xw != extra_writes_.end())
      for (int t : xw->second) {
        const int r = views_[t].root;
        used[r] = 1;
        if (def[r] < 0 || i < def[r]) def[r] = i;
        bump_end(r, i);
      }
  }
  for (int t : pinned) used[t] = 1;
  if (P.loss >= 0) { pinned.insert(views_[P.loss].root); used[views_[P.loss].root] = 1; }

  std::map<std::string, int64_t> state_off;
  int64_t bump[AR_COUNT] = {};
  auto place = [&](int t, int arena, int64_t off) {
    loc_[t].arena = arena;
    loc_[t].off = off;
    auto bo = bytes_override_.find(t);
    loc_[t].bytes = bo != bytes_override_.end() ? bo->second : std::max<int64_t>(4, P.T[t].numel * 4);
  };
  auto bump_place = [&](int t, int arena) {
    place(t, arena, bump[arena]);
    bump[arena] += align256(loc_[t].bytes);
  };

  const bool flat_m = adam_fused_ || (sgd_fused_ && sgd_.momentum > 0);
  std::set<int> grad_placed;
  grad_copy_.clear();
  grad_ready_.clear();
  for (int i = 0; i < nO; ++i) {
    const std::string& k = P.kind[i];
    int t = P.out[i];
    if (k == "param_input") {
      if (!parent) place(t, AR_PARAM, param_off_.at(P.op(i)["name"].str()));
      else loc_[t].arena = -2;  // resolved to the parent's arena
    } else if (k == "state_input") {
      const std::string& n = P.op(i)["name"].str();
      std::string pn;
      int arena = -1;
      if (adam_fused_ && n.rfind("adam_m_", 0) == 0) { pn = n.substr(7); arena = AR_M; }
      else if (adam_fused_ && n.rfind("adam_v_", 0) == 0) { pn = n.substr(7); arena = AR_V; }
      else if (sgd_fused_ && n.rfind("sgd_v_", 0) == 0) { pn = n.substr(6); arena = AR_M; }
      if (arena >= 0 && param_off_.count(pn)) place(t, arena, param_off_[pn]);
      else bump_place(t, AR_STATE);
    } else if (k == "tensor_input") {
      bump_place(t, AR_INPUT);
    } else if (is_const_kind(k)) {
      bump_place(t, AR_CONST);
    }
  }
  // Gradients go to the flat gradient arena (in place when the producing op
  // can write there directly, else by a copy before the optimizer section).
  for (auto& g : P.grads) {
    int G = g.second;
    int64_t off = param_off_.at(g.first);
    // The gradient is usually a same-shape view (sum_to_shape, reshape) of
    // the tensor its producer writes: place that root in the gradient slot.
    const TView& vg = views_[G];
    const int R = vg.onehot ? -1 : vg.root;
    bool direct = R >= 0 && vg.off == 0 && vg.contiguous && P.T[R].numel == P.T[G].numel &&
                  P.producer[R] >= 0 && !is_leaf_kind(P.kind[P.producer[R]]) &&
                  !is_const_kind(P.kind[P.producer[R]]) && loc_[R].arena < 0 && !grad_placed.count(R) &&
                  (!op_done_[P.producer[R]] || wt_reds_.count(P.producer[R])) && !ew_is_absorbed(P.producer[R]);
    if (direct) {
      place(R, AR_GRAD, off);
      grad_placed.insert(R);
      grad_ready_.push_back({g.first, std::max(end_bwd[R], def[R])});
    } else {
      grad_ready_.push_back({g.first, opt_stop});
      grad_copy_.push_back({G, off});
      int r = views_[G].onehot ? views_[views_[G].onehot_idx].root : views_[G].root;
      pinned.insert(r);
      used[r] = 1;
    }
  }
  // Pinned and temporaries.
  std::vector<int> temps;
  for (int t = 0; t < nT; ++t) {
    if (views_[t].root != t || views_[t].onehot || loc_[t].arena != -1 || !used[t]) continue;
    if (pinned.count(t)) bump_place(t, AR_PERSIST);
    else temps.push_back(t);
  }
  // Liveness packing of temporaries: intervals [def, end] by op index; an
  // op's output never shares storage with any of its live inputs.
  struct Blk { int64_t off, bytes; int d, e; };
  std::vector<Blk> blocks;
  std::sort(temps.begin(), temps.end(), [&](int a, int b) { return def[a] < def[b]; });
  int64_t temp_top = 0;
  for (int t : temps) {
    int64_t bytes = align256(std::max<int64_t>(4, P.T[t].numel * 4));
    int d = def[t] < 0 ? 0 : def[t], e = std::max(end[t], d);
    std::vector<std::pair<int64_t, int64_t>> busy;
    for (auto& b : blocks) if (!(b.e < d || b.d > e)) busy.emplace_back(b.off, b.off + b.bytes);
    std::sort(busy.begin(), busy.end());
    int64_t best = -1, best_gap = INT64_MAX, cur = 0;
    for (auto& b : busy) {
      if (b.first - cur >= bytes && b.first - cur < best_gap) { best = cur; best_gap = b.first - cur; }
      cur = std::max(cur, b.second);
    }
    if (best < 0) best = cur;
    place(t, AR_TEMP, best);
    blocks.push_back({best, bytes, d, e});
    temp_top = std::max(temp_top, best + bytes);
  }
  // Self-check: no two temporaries that share bytes are live at once.
  for (size_t i = 0; i < blocks.size(); ++i)
    for (size_t j = i + 1; j < blocks.size(); ++j) {
      const Blk& a = blocks[i]; const Blk& b = blocks[j];
      bool overlap_mem = a.off < b.off + b.bytes && b.off < a.off + a.bytes;
      bool overlap_time = !(a.e < b.d || b.e < a.d);
      if (overlap_mem && overlap_time) throw TgError("Error", "planner: temporary storage lifetime overlap");
    }
  bump[AR_TEMP] = temp_top;
  for (int i = 0; i < nO; ++i)
    if (!op_done_[i] || wt_reds_.count(i)) scratch_bytes_ = std::max(scratch_bytes_, scratch_for(P, i, action_[i]));
  bump[AR_SCRATCH] = align256(scratch_bytes_);
  if (!parent) {
    bump[AR_PARAM] = flat_floats_ * 4;
    if (!P.grads.empty()) bump[AR_GRAD] = flat_floats_ * 4;
    if (flat_m) bump[AR_M] = flat_floats_ * 4;
    if (adam_fused_) bump[AR_V] = flat_floats_ * 4;
  }
  bump[AR_PERSIST] += 256;  // data-parallel loss average slot
  loss_avg_off_ = bump[AR_PERSIST] - 256;
  for (int a = 0; a < AR_COUNT; ++a) {
    arena_bytes_[a] = bump[a];
    if (bump[a] > 0) {
      if (ctx->dry) {
        // placeholder, 1 TiB apart per arena: only addresses are computed
        arena_[a] = reinterpret_cast<void*>((uintptr_t)(a + 1) << 40);
        continue;
      }
      TG_CUDA(cudaMalloc(&arena_[a], (size_t)bump[a]));
      arena_owned_[a] = true;
      // On the context's stream: it is non-blocking, so a clear on the legacy
      // default stream would be unordered with the uploads and steps after it.
      TG_CUDA(cudaMemsetAsync(arena_[a], 0, (size_t)bump[a], ctx->stream));
    }
  }
  if (parent) {
    const Graph* g = parent;
    while (g->parent) g = g->parent;
    arena_[AR_PARAM] = g->arena_[AR_PARAM];
    arena_owned_[AR_PARAM] = false;
    for (auto& p : P.params) {
      auto it = g->param_off_.find(p.first);
      if (it == g->param_off_.end())
        throw TgError("Error", "forward graph references param '" + p.first + "' the parent does not have");
      place(p.second, AR_PARAM, it->second);
    }
  }
  if (ctx->dry) return;
  // State init values
  for (auto& s : P.states) {
    int t = s.tensor;
    if (s.init != 0.0 && loc_[t].arena >= 0) {
      float v = (float)s.init;
      uint32_t bits;
      memcpy(&bits, &v, 4);
      launch_fill(ptr(t), P.T[t].numel, bits, ctx->stream);
    }
  }
  TG_CUDA(cudaStreamSynchronize(ctx->stream));
}

void Graph::init_constants() {
  cudaStream_t s = ctx->stream;
  for (size_t i = 0; i < P.ops.size(); ++i) {
    const std::string& k = P.kind[i];
    int t = P.out[i];
    if (!is_const_kind(k) || loc_[t].arena < 0) continue;
    if (k == "arange") {
      launch_arange(ptr(t), P.T[t].numel, P.T[t].dtype, s);
    } else {
      double v = P.op(i)["value"].num();
      uint32_t bits;
      if (P.T[t].dtype == F32) { float f = (float)v; memcpy(&bits, &f, 4); }
      else { int32_t x = (int32_t)v; memcpy(&bits, &x, 4); }
      launch_fill(ptr(t), P.T[t].numel, bits, s);
    }
  }
  TG_CUDA(cudaStreamSynchronize(s));
  TG_CUDA(cudaGetLastError());
}

// ------------------------------------------------------------ emission ----
namespace {

struct EwBuilder {
  EwProgram p{};
  int nreg = 0;
  EwBuilder() { p.n_in = 0; p.n_out = 0; p.n_instr = 0; }
  int load(const EwInput& in) {
    if (p.n_in >= EW_MAX_IN) throw TgError("Error", "elementwise program: too many inputs");
    p.in[p.n_in] = in;
    int r = nreg++;
    EwInstr I{};
    I.op = EW_LOAD; I.dst = (uint8_t)r; I.a = (uint8_t)p.n_in;
    p.code[p.n_instr++] = I;
    p.n_in++;
    return r;
  }
  int emit(EwInstr I) {
    I.dst = (uint8_t)nreg++;
    if (nreg > EW_NREG || p.n_instr >= EW_MAX_INSTR) throw TgError("Error", "elementwise program too long");
    p.code[p.n_instr++] = I;
    return I.dst;
  }
};

}  // namespace

static bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

EwInput Graph::ew_input(int t, const std::vector<int64_t>& oshape, bool& vec_ok, bool with_ptr) {
  EwInput in{};
  const TView& v = views_[t];
  const auto& ts = P.T[t].shape;
  in.dtype = P.T[t].dtype;
  int R = (int)oshape.size(), rd = R - (int)ts.size();
  if (v.onehot) {
    if (ts != oshape) throw TgError("Error", "internal: virtual one-hot read with broadcast");
    in.mode = IN_ONEHOT;
    in.ptr = with_ptr ? ptr(v.onehot_idx) : nullptr;
    in.period = ts.back();
    return in;
  }
  in.ptr = with_ptr ? ptr(t) : nullptr;
  if (P.T[t].numel == 1) { in.mode = IN_SCALAR; return in; }
  std::vector<int64_t> pt(R, 1);
  for (size_t i = 0; i < ts.size(); ++i) pt[rd + i] = ts[i];
  if (v.contiguous) {
    if (pt == oshape) { in.mode = IN_FULL; if (!aligned16(in.ptr)) vec_ok = false; return in; }
    // suffix broadcast
    int k = 0;
    while (k < R && pt[k] == 1) ++k;
    bool suffix = true;
    for (int i = k; i < R; ++i) if (pt[i] != oshape[i]) suffix = false;
    if (suffix) {
      in.mode = IN_PERIOD; in.period = P.T[t].numel;
      if (in.period % 4 || !aligned16(in.ptr)) vec_ok = false;
      return in;
    }
    // prefix (trailing size-1 axes)
    int j = R;
    while (j > 0 && pt[j - 1] == 1) --j;
    bool prefix = true;
    for (int i = 0; i < j; ++i) if (pt[i] != oshape[i]) prefix = false;
    if (prefix) {
      int64_t per = 1;
      for (int i = j; i < R; ++i) per *= oshape[i];
      in.mode = IN_ROWDIV; in.period = per;
      if (per % 4) vec_ok = false;
      return in;
    }
  }
  if (R > EW_MAX_RANK) throw TgError("Error", "elementwise op rank > 6 with a strided operand");
  in.mode = IN_STRIDED;
  for (int i = 0; i < R; ++i) {
    if (i < rd) in.strides[i] = 0;
    else in.strides[i] = (pt[i] == 1 && oshape[i] != 1) ? 0 : v.strides[i - rd];
  }
  vec_ok = false;
  return in;
}

// Tensors that are exactly zero above the diagonal of their last two dims:
// a causal softmax's result (the masked entries are written as 0), and
// dropouts, scalings and same-shape products of such a tensor (0 times a
// finite value stays 0).
bool Graph::causal_zero(int t) {
  auto it = causal_memo_.find(t);
  if (it != causal_memo_.end()) return it->second;
  causal_memo_[t] = false;
  bool z = false;
  const int p = P.producer[t];
  if (p >= 0) {
    const std::string& k = P.kind[p];
    const auto& O = P.op(p);
    if (k == "softmax_causal_last") z = true;
    else if (k == "dropout" || k == "mul_scalar" ||
             ((k == "reshape" || k == "stop_gradient") && P.T[O["a"].i32()].shape == P.T[t].shape))
      z = causal_zero(O["a"].i32());
    else if (k == "mul") {
      for (const char* f : {"a", "b"}) {
        const int x = O[f].i32();
        if (P.T[x].shape == P.T[t].shape && causal_zero(x)) z = true;
      }
    }
  }
  causal_memo_[t] = z;
  return z;
}

double Graph::tensor_bytes(int t) const {
  const TView& v = views_[t];
  if (v.onehot) return 4.0 * (double)P.T[v.onehot_idx].numel;  // a virtual one-hot reads its indices
  return 4.0 * (double)P.T[t].numel;
}

void Graph::emit_launches() {
  launches_.clear();
  launch_kind_.clear();
  launch_bytes_.clear();
  next_bytes_ = 0;
  post_.clear();
  const int nO = (int)P.ops.size();
  float* scratch = reinterpret_cast<float*>(arena_[AR_SCRATCH]);
  size_t scratch_floats = (size_t)(arena_bytes_[AR_SCRATCH] / 4);
  const int* seed_ptr = nullptr;
  auto it_seed = P.inputs.find("__prngSeed");
  if (it_seed != P.inputs.end()) seed_ptr = reinterpret_cast<const int*>(ptr(it_seed->second));

  auto add = [&](const std::string& kind, std::function<void(cudaStream_t)> f) {
    launches_.push_back(std::move(f));
    launch_kind_.push_back(kind);
    launch_bytes_.push_back(next_bytes_);
    next_bytes_ = 0;
  };

  auto mk_input = [&](int t, const std::vector<int64_t>& oshape, bool& vec_ok) -> EwInput {
    return ew_input(t, oshape, vec_ok);
  };

  auto finish_ew = [&](EwBuilder& B, int out_t, int out_reg, bool vec_ok, const std::string& kind) {
    const auto& os = P.T[out_t].shape;
    B.p.numel = P.T[out_t].numel;
    B.p.rank = (int)os.size();
    for (int i = 0; i < B.p.rank && i < EW_MAX_RANK; ++i) B.p.dims[i] = os[i];
    B.p.out[0] = ptr(out_t);
    B.p.out_reg[0] = (uint8_t)out_reg;
    B.p.n_out = 1;
    B.p.seed = seed_ptr;
    B.p.drop_offset = (int64_t)ctx->rank * B.p.numel;
    B.p.vec4 = vec_ok && (B.p.numel % 4 == 0) && aligned16(B.p.out[0]) ? 1 : 0;
    EwProgram prog = B.p;
    add(kind, [prog](cudaStream_t s) { launch_ew(prog, s); });
  };

  auto emit_copy = [&](int in_t, int64_t in_extra_off, const std::vector<int64_t>& dims,
                       const std::vector<int64_t>& in_strides, void* out, const std::vector<int64_t>& out_strides,
                       const std::string& kind) {
    if ((int)dims.size() > CP_MAX_RANK) throw TgError("Error", "copy rank > 8");
    CopyDesc d{};
    d.rank = (int)dims.size();
    d.numel = 1;
    for (int i = 0; i < d.rank; ++i) {
      d.dims[i] = dims[i]; d.in_strides[i] = in_strides[i]; d.out_strides[i] = out_strides[i]; d.numel *= dims[i];
    }
    const char* src = reinterpret_cast<const char*>(ptr(in_t)) + in_extra_off * 4;
    add(kind, [d, src, out](cudaStream_t s) { launch_copy(d, src, out, s); });
  };

  auto ensure_contig = [&](int t, const char* what) {
    if (!is_contig(t)) throw TgError("Error", std::string("internal: ") + what + " expects a contiguous operand");
  };

  const bool dp = ctx->world > 1 && !parent && (adam_fused_ || sgd_fused_);
  // Data parallel: gradient buckets. Once the ops that last touch a group of
  // gradients (in backward order) have been emitted and the group holds
  // DP_BUCKET_BYTES, a launch forks the communication stream off the step's
  // stream and allreduces those ranges there, overlapping the rest of the
  // backward pass; the optimizer section starts after a join. Every rank
  // plans the same launch list, so the collectives are issued in the same
  // order everywhere.
  static const int64_t DP_BUCKET_BYTES = [] {
    const char* e = getenv("TG_DP_BUCKET_MB");  // bucket size override (tests, tuning)
    return e ? std::max<int64_t>(256, (int64_t)(atof(e) * 1048576.0)) : (int64_t)(24ll << 20);
  }();
  std::vector<std::pair<int, int64_t>> dp_order;  // (ready op, byte offset) per gradient
  std::map<int64_t, int64_t> dp_bytes;            // byte offset -> padded bytes
  if (dp) {
    std::map<std::string, int> grad_of;
    for (auto& g : P.grads) grad_of[g.first] = g.second;
    for (auto& gr : grad_ready_) {
      const int64_t off = param_off_.at(gr.first);
      dp_order.push_back({gr.second, off});
      const int G = grad_of.at(gr.first);
      dp_bytes[off] = (P.T[G].numel + 63) / 64 * 64 * 4;
    }
    std::sort(dp_order.begin(), dp_order.end());
    for (auto e : dp_events_) cudaEventDestroy(e);
    dp_events_.clear();
  }
  size_t dp_next = 0;
  std::vector<int64_t> dp_pending;
  int64_t dp_pending_bytes = 0;
  auto dp_flush = [&]() {
    if (dp_pending.empty()) return;
    std::sort(dp_pending.begin(), dp_pending.end());
    std::vector<std::pair<float*, int64_t>> ranges;  // merged adjacent ranges, in floats
    for (int64_t off : dp_pending) {
      float* p = reinterpret_cast<float*>(reinterpret_cast<char*>(arena_[AR_GRAD]) + off);
      const int64_t n = dp_bytes[off] / 4;
      if (!ranges.empty() && ranges.back().first + ranges.back().second == p) ranges.back().second += n;
      else ranges.push_back({p, n});
    }
    dp_pending.clear();
    dp_pending_bytes = 0;
    cudaEvent_t ev = nullptr;
    if (!ctx->dry) TG_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    dp_events_.push_back(ev);
    Context* c = ctx;
    int64_t tot = 0;
    for (auto& r : ranges) tot += r.second;
    add("nccl_allreduce|bucket floats=" + std::to_string(tot) + " ranges=" + std::to_string(ranges.size()),
        [c, ev, ranges](cudaStream_t s) {
          TG_CUDA(cudaEventRecord(ev, s));
          TG_CUDA(cudaStreamWaitEvent(c->comm_stream, ev, 0));
          c->allreduce_ranges(ranges, c->comm_stream);
        });
  };
  auto dp_collect = [&](int upto, bool all) {
    while (dp_next < dp_order.size() && (all || dp_order[dp_next].first < upto)) {
      dp_pending.push_back(dp_order[dp_next].second);
      dp_pending_bytes += dp_bytes[dp_order[dp_next].second];
      ++dp_next;
    }
    if (dp_pending_bytes >= DP_BUCKET_BYTES || all) dp_flush();
  };
  for (int i = 0; i <= nO; ++i) {
    if (dp && i < P.opt_start) dp_collect(i, false);
    if (i == P.opt_start && !parent && !P.grads.empty()) {
      for (auto& gc : grad_copy_) {
        int G = gc.first;
        float* dst = reinterpret_cast<float*>(reinterpret_cast<char*>(arena_[AR_GRAD]) + gc.second);
        if (views_[G].onehot) throw TgError("Error", "internal: one-hot gradient");
        auto dims = P.T[G].shape;
        emit_copy(G, 0, dims, views_[G].strides, dst, cstrides(dims), "grad_copy");
      }
      if (dp) {
        dp_collect(i, true);
        cudaEvent_t join = nullptr;
        if (!ctx->dry) TG_CUDA(cudaEventCreateWithFlags(&join, cudaEventDisableTiming));
        dp_events_.push_back(join);
        Context* c = ctx;
        add("nccl_join", [c, join](cudaStream_t s) {
          TG_CUDA(cudaEventRecord(join, c->comm_stream));
          TG_CUDA(cudaStreamWaitEvent(s, join, 0));
        });
      }
    }
    if (i == nO) break;
    if (op_done_[i]) continue;
    if (ew_is_absorbed(i)) continue;
    if (ew_group_of(i) >= 0) {
      emit_ew_group(ew_group_of(i), seed_ptr, scratch, scratch_floats, add);
      continue;
    }
    const std::string& k = P.kind[i];
    const auto& O = P.op(i);
    int o = P.out[i];
    const auto& os = P.T[o].shape;
    next_bytes_ = 0;
    if (ew_kinds().count(k) || k == "reshape" || k == "stop_gradient" || k == "sum_to_shape" || k == "permute" ||
        k == "mean_last" || k == "sum_last" || k == "max_last" || k == "argmax_last" || k == "log_softmax_last" ||
        k == "softmax_causal_last" || k == "categorical_last") {
      std::set<int> rd;
      if (ew_kinds().count(k)) for (int t : ew_operands(P, i)) rd.insert(t);
      else rd.insert(O["a"].i32());
      for (int t : rd) next_bytes_ += tensor_bytes(t);
      next_bytes_ += tensor_bytes(o);
      auto sd = softmax_drop_.find(i);
      if (sd != softmax_drop_.end()) next_bytes_ += tensor_bytes(P.out[sd->second]);
    }
    if (action_[i] == 110 || action_[i] == 111) {
      const AttnBlock& A = attn_[attn_of_.at(i)];
      auto aview = [&](int t, bool swap_last) {
        const TView& v = views_[t];
        AttnView a{reinterpret_cast<float*>(ptr(t)), v.strides[0], v.strides[1], v.strides[2], v.strides[3]};
        if (swap_last) std::swap(a.s2, a.s3);
        return a;
      };
      const auto& qs = P.T[A.q].shape;
      AttnParams ap{};
      ap.B = (int)qs[0]; ap.H = (int)qs[1]; ap.T = (int)qs[2]; ap.D = (int)qs[3];
      ap.q = aview(A.q, false); ap.k = aview(A.k, false); ap.v = aview(A.v, false); ap.o = aview(A.o, false);
      ap.ml = reinterpret_cast<float*>(ptr(A.ml));
      ap.scale = A.scale; ap.p = A.p; ap.keep_scale = A.keep_scale; ap.salt = A.salt;
      ap.dropout = A.dropout ? 1 : 0;
      ap.seed = A.dropout ? seed_ptr : nullptr;
      ap.drop_off = (int64_t)ctx->rank * P.T[A.p_t].numel;
      char label[96];
      snprintf(label, sizeof label, "%s|B=%d H=%d T=%d D=%d", action_[i] == 110 ? "attn_fwd" : "attn_bwd", ap.B, ap.H,
               ap.T, ap.D);
      if (action_[i] == 110) {
        add(label, [ap](cudaStream_t s) { launch_attn_fwd(ap, s); });
      } else {
        ap.dout = aview(A.dout, false);
        ap.dq = aview(A.dq, false);
        ap.dk = aview(A.dkt, true);
        ap.dv = aview(A.dv, false);
        ap.dv_row = reinterpret_cast<float*>(ptr(A.rowdot));
        ap.ds = reinterpret_cast<float*>(ptr(A.ds));
        ap.ds_ld = ap.T;
        add(label, [ap](cudaStream_t s) { launch_attn_bwd(ap, s); });
      }
      continue;
    }
    if (action_[i] == 103) {
      const int m = P.producer[O["a"].i32()];
      int u = P.op(m)["a"].i32(), oh = P.op(m)["b"].i32();
      if (!views_[oh].onehot) std::swap(u, oh);
      const int idx = P.op(P.producer[oh])["indices"].i32(), g = P.op(P.producer[u])["a"].i32();
      const int64_t V = P.T[oh].shape.back(), rows = P.T[o].numel;
      const float* gp = reinterpret_cast<const float*>(ptr(g));
      const int* ip = reinterpret_cast<const int*>(ptr(idx));
      float* op = reinterpret_cast<float*>(ptr(o));
      next_bytes_ = 4.0 * (double)(P.T[g].numel + P.T[idx].numel + P.T[o].numel);
      add("row_hit", [=](cudaStream_t s) { launch_row_hit(gp, ip, op, rows, V, s); });
      continue;
    }
    if (action_[i] == 102) {
      const int m = P.producer[O["a"].i32()];
      int x = P.op(m)["a"].i32(), oh = P.op(m)["b"].i32();
      if (!views_[oh].onehot) std::swap(x, oh);
      const int idx = P.op(P.producer[oh])["indices"].i32();
      const int64_t V = P.T[x].shape.back(), rows = P.T[o].numel;
      const float* xp = reinterpret_cast<const float*>(ptr(x));
      const int* ip = reinterpret_cast<const int*>(ptr(idx));
      float* op = reinterpret_cast<float*>(ptr(o));
      next_bytes_ = 4.0 * (double)(rows + P.T[idx].numel + P.T[o].numel);  // one element read per row
      add("pick", [=](cudaStream_t s) { launch_pick(xp, ip, op, rows, V, s); });
      continue;
    }
    if (action_[i] == 100) {
      int a = O["a"].i32(), b = O["b"].i32();
      int idx = P.op(P.producer[a])["indices"].i32();
      ensure_contig(b, "embedding table");
      int64_t V = P.T[b].shape[0], D = P.T[b].shape[1], rows = P.T[idx].numel;
      const int* ip = reinterpret_cast<const int*>(ptr(idx));
      const float* tp = reinterpret_cast<const float*>(ptr(b));
      float* op = reinterpret_cast<float*>(ptr(o));
      next_bytes_ = 4.0 * (double)(rows + 2 * rows * D);  // indices, gathered rows, output
      add("gather_rows", [=](cudaStream_t s) { launch_gather_rows(ip, tp, op, rows, V, D, s); });
      continue;
    }
    if (action_[i] == 101) {
      int a = O["a"].i32(), b = O["b"].i32();
      int oh = P.op(P.producer[P.op(P.producer[a])["a"].i32()])["a"].i32();
      int idx = P.op(P.producer[oh])["indices"].i32();
      ensure_contig(b, "embedding grad");
      int64_t V = P.T[a].shape[0], rows = P.T[b].shape[0], D = P.T[b].shape[1];
      const int* ip = reinterpret_cast<const int*>(ptr(idx));
      const float* dyp = reinterpret_cast<const float*>(ptr(b));
      float* op = reinterpret_cast<float*>(ptr(o));
      int* scr = reinterpret_cast<int*>(scratch);
      next_bytes_ = 4.0 * (double)(rows + rows * D + V * D);  // indices, row gradients, table gradient
      add("embedding_grad", [=](cudaStream_t s) { launch_embedding_grad(ip, dyp, op, rows, V, D, scr, s); });
      continue;
    }
    // ---------------------------------------------------- elementwise --
    static const std::map<std::string, int> bin = {{"add", EW_ADD}, {"sub", EW_SUB}, {"mul", EW_MUL},
                                                   {"div", EW_DIV}, {"min", EW_MIN}, {"max", EW_MAX}};
    static const std::map<std::string, int> un = {
        {"sqrt", EW_SQRT}, {"rsqrt", EW_RSQRT}, {"log", EW_LOG}, {"exp", EW_EXP}, {"relu", EW_RELU},
        {"neg", EW_NEG}, {"abs", EW_ABS}, {"tanh", EW_TANH}, {"sigmoid", EW_SIGMOID}, {"erf", EW_ERF},
        {"sin", EW_SIN}, {"cos", EW_COS}};
    bool vec_ok = true;
    if (bin.count(k) || k == "less" || k == "greater") {
      if (bin.count(k) && P.T[o].dtype != F32) throw TgError("Error", k + ": only f32 arithmetic is supported");
      EwBuilder B;
      int ra = B.load(mk_input(O["a"].i32(), os, vec_ok));
      int rb = B.load(mk_input(O["b"].i32(), os, vec_ok));
      EwInstr I{};
      I.op = (uint8_t)(bin.count(k) ? bin.at(k) : (k == "less" ? EW_LESS : EW_GREATER));
      I.a = (uint8_t)ra; I.b = (uint8_t)rb;
      I.aux = (P.T[O["a"].i32()].dtype != F32) ? 1u : 0u;
      finish_ew(B, o, B.emit(I), vec_ok, k);
      continue;
    }
    if (un.count(k) || k == "mul_scalar" || k == "add_scalar" || k == "where_causal" || k == "dropout" ||
        k == "broadcast_to" || ((k == "reshape" || k == "stop_gradient" || k == "sum_to_shape") &&
                                P.T[o].numel == P.T[O["a"].i32()].numel && is_contig(O["a"].i32()))) {
      EwBuilder B;
      int ra = B.load(mk_input(O["a"].i32(), (k == "reshape" || k == "stop_gradient" || k == "sum_to_shape")
                                                  ? P.T[O["a"].i32()].shape : os, vec_ok));
      if (k == "reshape" || k == "stop_gradient" || k == "sum_to_shape") {
        // materialised identity copy (the output is observable, so it owns storage)
        B.p.numel = P.T[o].numel;
        EwProgram& pp = B.p;
        pp.rank = 1; pp.dims[0] = pp.numel;
        pp.in[0].mode = IN_FULL;
        pp.out[0] = ptr(o); pp.out_reg[0] = (uint8_t)ra; pp.n_out = 1;
        pp.vec4 = (pp.numel % 4 == 0 && aligned16(pp.out[0]) && aligned16(pp.in[0].ptr)) ? 1 : 0;
        EwProgram prog = pp;
        add(k, [prog](cudaStream_t s) { launch_ew(prog, s); });
        continue;
      }
      int rout = ra;
      if (k != "broadcast_to") {
        EwInstr I{};
        I.a = (uint8_t)ra;
        if (un.count(k)) I.op = (uint8_t)un.at(k);
        else if (k == "mul_scalar") { I.op = EW_MULS; I.imm = (float)O["scalar"].num(); }
        else if (k == "add_scalar") { I.op = EW_ADDS; I.imm = (float)O["scalar"].num(); }
        else if (k == "where_causal") { I.op = EW_WHERE_CAUSAL; I.aux = (uint32_t)os.back(); I.imm = (float)O["fillValue"].num(); }
        else {
          I.op = EW_DROPOUT;
          double p = O["p"].num();
          I.imm = f32_lit8(p);
          I.imm2 = f32_lit8(1.0 / (1.0 - p));
          I.aux = (uint32_t)(((uint64_t)O["salt"].i64() * 0x9E3779B1ull) & 0xFFFFFFFFull);
        }
        rout = B.emit(I);
      }
      finish_ew(B, o, rout, vec_ok, k);
      continue;
    }
    if (k == "where") {
      EwBuilder B;
      int rc = B.load(mk_input(O["cond"].i32(), os, vec_ok));
      int ra = B.load(mk_input(O["a"].i32(), os, vec_ok));
      int rb = B.load(mk_input(O["b"].i32(), os, vec_ok));
      EwInstr I{};
      I.op = EW_WHERE; I.a = (uint8_t)rc; I.b = (uint8_t)ra; I.c = (uint8_t)rb;
      finish_ew(B, o, B.emit(I), vec_ok, k);
      continue;
    }
    if (k == "relu_grad") {
      EwBuilder B;
      int rx = B.load(mk_input(O["x"].i32(), os, vec_ok));
      int rd = B.load(mk_input(O["dy"].i32(), os, vec_ok));
      EwInstr I{};
      I.op = EW_RELU_GRAD; I.a = (uint8_t)rx; I.b = (uint8_t)rd;
      finish_ew(B, o, B.emit(I), vec_ok, k);
      continue;
    }
    if (k == "adam_update_m" || k == "adam_update_v") {
      EwBuilder B;
      bool isM = k == "adam_update_m";
      int r0 = B.load(mk_input(O[isM ? "m" : "v"].i32(), os, vec_ok));
      int r1 = B.load(mk_input(O["g"].i32(), os, vec_ok));
      double beta = O[isM ? "beta1" : "beta2"].num();
      EwInstr I{};
      I.op = isM ? EW_ADAM_M : EW_ADAM_V; I.a = (uint8_t)r0; I.b = (uint8_t)r1;
      I.imm = (float)beta; I.imm2 = (float)(1.0 - beta);
      finish_ew(B, o, B.emit(I), vec_ok, k);
      continue;
    }
    if (k == "adam_update_p") {
      EwBuilder B;
      int rp = B.load(mk_input(O["p"].i32(), os, vec_ok));
      int rm = B.load(mk_input(O["mNew"].i32(), os, vec_ok));
      int rl = B.load(mk_input(O["lrt"].i32(), os, vec_ok));
      int rs;
      if (!O["decayShrinkTensor"].is_null()) rs = B.load(mk_input(O["decayShrinkTensor"].i32(), os, vec_ok));
      else { EwInstr C{}; C.op = EW_CONST; C.imm = (float)O["decayShrink"].num(); rs = B.emit(C); }
      int rv = B.load(mk_input(O["vNew"].i32(), os, vec_ok));
      EwInstr I{};
      I.op = EW_ADAM_P; I.a = (uint8_t)rp; I.b = (uint8_t)rm; I.c = (uint8_t)rl; I.d = (uint8_t)rs; I.e = (uint8_t)rv;
      I.imm = (float)O["eps"].num();
      finish_ew(B, o, B.emit(I), vec_ok, k);
      continue;
    }
    // ------------------------------------------------------------ rows --
    if (k == "sum_last" || k == "mean_last" || k == "argmax_last" || k == "log_softmax_last" ||
        k == "softmax_causal_last" || k == "categorical_last") {
      int a = O["a"].i32();
      ensure_contig(a, k.c_str());
      int64_t D = P.T[a].shape.back(), rows = P.T[a].numel / std::max<int64_t>(D, 1);
      int kind = k == "sum_last" ? ROW_SUM : k == "mean_last" ? ROW_MEAN : k == "argmax_last" ? ROW_ARGMAX
               : k == "log_softmax_last" ? ROW_LOGSOFTMAX : k == "softmax_causal_last" ? ROW_SOFTMAX_CAUSAL
               : ROW_CATEGORICAL;
      const float* x = reinterpret_cast<const float*>(ptr(a));
      void* out = ptr(o);
      const int* sd = k == "categorical_last" ? reinterpret_cast<const int*>(ptr(O["seed"].i32())) : nullptr;
      uint32_t salt = k == "categorical_last" ? (uint32_t)(((uint64_t)O["salt"].i64() * 0x9E3779B1ull) & 0xFFFFFFFFull) : 0;
      auto sdrop = softmax_drop_.find(i);
      if (sdrop != softmax_drop_.end()) {  // the softmax also writes its dropout
        const auto& DO = P.op(sdrop->second);
        const double pd = DO["p"].num();
        RowDropout rd{};
        rd.out2 = reinterpret_cast<float*>(ptr(P.out[sdrop->second]));
        rd.seed = seed_ptr;
        rd.salt = (uint32_t)(((uint64_t)DO["salt"].i64() * 0x9E3779B1ull) & 0xFFFFFFFFull);
        rd.p = f32_lit8(pd);
        rd.keep_scale = f32_lit8(1.0 / (1.0 - pd));
        rd.drop_off = (int64_t)ctx->rank * P.T[o].numel;
        float* fo = reinterpret_cast<float*>(out);
        add("softmax_causal_last+dropout", [=](cudaStream_t s) { launch_softmax_causal_dropout(x, fo, rows, D, rd, s); });
        continue;
      }
      add(k, [=](cudaStream_t s) { launch_row(kind, x, out, rows, D, s, sd, salt, scratch, scratch_floats); });
      continue;
    }
    if (k == "sum_to_shape") {
      int a = O["a"].i32();
      ensure_contig(a, "sum_to_shape");
      const auto& is = P.T[a].shape;
      int R = (int)is.size(), rd = R - (int)os.size();
      std::vector<int64_t> keep(R, 0);
      for (int d = 0; d < R; ++d) keep[d] = (d >= rd && !(os[d - rd] == 1 && is[d] != 1)) ? 1 : 0;
      bool suffix = true;
      bool seen_keep = false;
      for (int d = 0; d < R; ++d) { if (keep[d]) seen_keep = true; else if (seen_keep && is[d] != 1) suffix = false; }
      // kept dims all before the reduced ones: a row sum over the trailing extent
      bool prefix = true;
      bool seen_red = false;
      for (int d = 0; d < R; ++d) {
        if (is[d] == 1) continue;
        if (!keep[d]) seen_red = true; else if (seen_red) prefix = false;
      }
      if (prefix && !suffix) {
        const float* x = reinterpret_cast<const float*>(ptr(a));
        float* out = reinterpret_cast<float*>(ptr(o));
        int64_t rows = P.T[o].numel, D = P.T[a].numel / std::max<int64_t>(rows, 1);
        add("rowsum", [=](cudaStream_t s) { launch_row(ROW_SUM, x, out, rows, D, s, nullptr, 0, scratch, scratch_floats); });
        continue;
      }
      const float* x = reinterpret_cast<const float*>(ptr(a));
      float* out = reinterpret_cast<float*>(ptr(o));
      int64_t inner = P.T[o].numel, outer = P.T[a].numel / std::max<int64_t>(inner, 1);
      if (suffix) {
        add("colsum", [=](cudaStream_t s) { launch_colsum(x, out, outer, inner, scratch, s); });
      } else if (mid_runs(is, keep, nullptr)) {
        int64_t r3[3];
        mid_runs(is, keep, r3);
        const int64_t R1 = r3[0], Km = r3[1], R2 = r3[2];
        add("sum_mid", [=](cudaStream_t s) { launch_sum_mid(x, out, R1, Km, R2, scratch, s); });
      } else {
        std::vector<int64_t> dims = is;
        int64_t in_n = P.T[a].numel, out_n = inner;
        add("sum_general", [=](cudaStream_t s) {
          launch_sum_general(x, out, (int)dims.size(), dims.data(), keep.data(), in_n, out_n, s);
        });
      }
      continue;
    }
    // ------------------------------------------------------------ GEMM --
    if (k == "matmul" || k == "matmul_batched") {
      int a = O["a"].i32(), b = O["b"].i32();
      const TView& va = views_[a];
      const TView& vb = views_[b];
      if (va.onehot || vb.onehot) throw TgError("Error", "internal: GEMM on a virtual one-hot");
      const auto& as = P.T[a].shape;
      const auto& bs = P.T[b].shape;
      int ra = (int)as.size(), rb = (int)bs.size();
      GemmDesc g{};
      g.K = as[ra - 1];
      g.N = bs[rb - 1];
      g.alpha = gemm_alpha_[i];
      g.A = reinterpret_cast<const float*>(ptr(a));
      g.B = reinterpret_cast<const float*>(ptr(b));
      g.C = reinterpret_cast<float*>(ptr(o));
      g.lda_m = va.strides[ra - 2]; g.lda_k = va.strides[ra - 1];
      g.ldb_k = vb.strides[rb - 2]; g.ldb_n = vb.strides[rb - 1];
      // C may be a strided view (written straight into a later permute's layout)
      const TView& vc = views_[o];
      const int rc = (int)os.size();
      g.ldc = vc.strides[rc - 2];
      g.ldc_n = vc.strides[rc - 1];
      g.batch2 = 1;
      std::vector<int64_t> bd(os.begin(), os.end() - 2), sa, sb, sc;
      int nb = (int)bd.size();
      for (int d = 0; d < nb; ++d) {
        sa.push_back(va.strides[d]);
        sb.push_back(k == "matmul" ? 0 : vb.strides[d]);
        sc.push_back(vc.strides[d]);
      }
      g.M = as[ra - 2];
      // matmul: fold leading dims into M when A's and C's layouts allow it
      if (k == "matmul") {
        bool fold = true;
        int64_t expect = g.lda_m * g.M, expect_c = g.ldc * g.M;
        for (int d = nb - 1; d >= 0; --d) {
          if (bd[d] != 1 && (sa[d] != expect || sc[d] != expect_c)) fold = false;
          expect *= bd[d]; expect_c *= bd[d];
        }
        if (fold) { int64_t m = g.M; for (auto x : bd) m *= x; g.M = m; bd.clear(); sa.clear(); sb.clear(); sc.clear(); nb = 0; }
      }
      // drop unit dims, merge adjacent batch dims that all three operands allow
      std::vector<int64_t> B2, SA, SB, SC;
      for (int d = 0; d < nb; ++d) if (bd[d] != 1) { B2.push_back(bd[d]); SA.push_back(sa[d]); SB.push_back(sb[d]); SC.push_back(sc[d]); }
      for (int d = (int)B2.size() - 2; d >= 0; --d) {
        if (SA[d] == SA[d + 1] * B2[d + 1] && SB[d] == SB[d + 1] * B2[d + 1] && SC[d] == SC[d + 1] * B2[d + 1]) {
          B2[d] *= B2[d + 1]; SA[d] = SA[d + 1]; SB[d] = SB[d + 1]; SC[d] = SC[d + 1];
          B2.erase(B2.begin() + d + 1); SA.erase(SA.begin() + d + 1); SB.erase(SB.begin() + d + 1); SC.erase(SC.begin() + d + 1);
        }
      }
      if (B2.size() > 2) throw TgError("Error", "matmul: operand layout needs more than two batch dims");
      if (B2.empty()) { g.batch = 1; }
      else if (B2.size() == 1) { g.batch = B2[0]; g.a_batch = SA[0]; g.b_batch = SB[0]; g.c_batch = SC[0]; }
      else {
        g.batch = B2[0] * B2[1]; g.batch2 = B2[1];
        g.a_batch = SA[0]; g.b_batch = SB[0]; g.c_batch = SC[0];
        g.a_batch2 = SA[1]; g.b_batch2 = SB[1]; g.c_batch2 = SC[1];
      }
      g.workspace = scratch;
      g.workspace_floats = (int64_t)scratch_floats;
      // causal A: the square [.., T, T] operand of attention's P.V and of the
      // gradient GEMMs, exactly zero above (or, transposed, below) the diagonal
      auto square_root = [&](const TView& v, int64_t T) {
        const auto& rs = P.T[v.root].shape;
        const int rr = (int)rs.size();
        return !v.onehot && v.off == 0 && rr >= 2 && rs[rr - 1] == T && rs[rr - 2] == T && causal_zero(v.root);
      };
      if (k == "matmul_batched" && g.M == g.K && g.M >= 256 && square_root(va, g.M)) {
        if (g.lda_m == g.M && g.lda_k == 1) g.tri = 1;
        else if (g.lda_m == 1 && g.lda_k == g.M) g.tri = 2;
      }
      if (k == "matmul_batched" && !g.tri && g.N == g.K && g.N >= 256 && square_root(vb, g.N)) {
        if (g.ldb_k == g.N && g.ldb_n == 1) g.tri_cols = 2;       // B(k, n) = R[k][n]: zero for n > k
        else if (g.ldb_k == 1 && g.ldb_n == g.N) g.tri_cols = 1;  // B(k, n) = R[n][k]: zero for k > n
      }
      // TMA needs 16-byte aligned bases and row strides. An operand whose
      // outer stride is not a multiple of 4 floats (a vocabulary of 65) is
      // first copied to padded rows after the split-K workspace, so the
      // contraction still runs on the tensor cores.
      struct Pad { const float* src; int64_t ld_src; float* dst; int64_t ld_dst, rows, cols; };
      std::vector<Pad> pads;
      if (g.batch == 1 && g.M * g.N * g.K >= (int64_t)64 * 64 * 64 && g.K >= 16) {
        const int64_t wsf = (gemm_tc_workspace_floats(g.M, g.N, g.K, 1) + 63) / 64 * 64;
        float* next = scratch + wsf;
        auto up4 = [](int64_t v) { return (v + 3) / 4 * 4; };
        auto stage = [&](const float*& p, int64_t& s_outer, int64_t s_inner, int64_t outer, int64_t inner) {
          if (s_inner != 1) return;
          if (s_outer % 4 == 0 && !(reinterpret_cast<uintptr_t>(p) & 15)) return;
          const int64_t ld = up4(inner);
          pads.push_back({p, s_outer, next, ld, outer, inner});
          p = next;
          s_outer = ld;
          next += (outer * ld + 63) / 64 * 64;
        };
        if (g.lda_k == 1) stage(g.A, g.lda_m, g.lda_k, g.M, g.K); else stage(g.A, g.lda_k, g.lda_m, g.K, g.M);
        if (g.ldb_k == 1) stage(g.B, g.ldb_n, g.ldb_k, g.N, g.K); else stage(g.B, g.ldb_k, g.ldb_n, g.K, g.N);
        if (next > scratch + scratch_floats) throw TgError("Error", "internal: scratch too small for GEMM staging");
        if (!pads.empty()) g.workspace_floats = wsf;
      }
      char label[160];
      snprintf(label, sizeof label, "%s|M=%lld N=%lld K=%lld b=%lld A%s B%s%s%s", k.c_str(), (long long)g.M,
               (long long)g.N, (long long)g.K, (long long)g.batch, g.lda_k == 1 ? "k" : "mn",
               g.ldb_k == 1 ? "k" : "mn", pads.empty() ? "" : " padded", (g.tri || g.tri_cols) ? " causal" : "");
      add(label, [g, pads](cudaStream_t s) {
        for (const Pad& p : pads) launch_pad_rows(p.src, p.ld_src, p.dst, p.ld_dst, p.rows, p.cols, s);
        if (!launch_gemm_tc(g, s)) launch_gemm_simt(g, s);
      });
      continue;
    }
    // ---------------------------------------------------------- layout --
    if (k == "permute" || k == "reshape" || k == "stop_gradient" || k == "slice_range") {
      int a = O["a"].i32();
      const TView& va = views_[a];
      if (va.onehot) throw TgError("Error", "internal: layout op on a virtual one-hot");
      std::vector<int64_t> in_str;
      int64_t extra = 0;
      if (k == "permute") {
        for (auto& pv : O["perm"].a) in_str.push_back(va.strides[pv.i32()]);
      } else if (k == "slice_range") {
        in_str = va.strides;
        extra = O["start"].i64() * va.strides[O["axis"].i32()];
      } else {
        if (!va.contiguous) throw TgError("Error", "internal: reshape of a strided view");
        in_str = cstrides(os);
      }
      emit_copy(a, extra, os, in_str, ptr(o), views_[o].strides, k);
      continue;
    }
    if (k == "concat") {
      int ax = O["axis"].i32();
      auto ocs = cstrides(os);
      int64_t cur = 0;
      for (auto& x : O["inputs"].a) {
        int t = x.i32();
        const auto& ts = P.T[t].shape;
        char* dst = reinterpret_cast<char*>(ptr(o)) + cur * ocs[ax] * 4;
        emit_copy(t, 0, ts, views_[t].strides, dst, ocs, "concat");
        cur += ts[ax];
      }
      continue;
    }
    if (k == "scatter_axis") {
      int a = O["a"].i32();
      void* op = ptr(o);
      int64_t n = P.T[o].numel;
      add("scatter_fill", [op, n](cudaStream_t s) { launch_fill(op, n, 0u, s); });
      auto ocs = cstrides(os);
      char* dst = reinterpret_cast<char*>(op) + O["start"].i64() * ocs[O["axis"].i32()] * 4;
      emit_copy(a, 0, P.T[a].shape, views_[a].strides, dst, ocs, "scatter_axis");
      continue;
    }
    if (k == "one_hot") {
      int idx = O["indices"].i32();
      const int* ip = reinterpret_cast<const int*>(ptr(idx));
      void* op = ptr(o);
      int64_t n = P.T[idx].numel, depth = O["depth"].i64();
      int dt = P.T[o].dtype;
      add("one_hot", [=](cudaStream_t s) { launch_one_hot(ip, op, n, depth, dt, s); });
      continue;
    }
    if (k == "randn") {
      float* op = reinterpret_cast<float*>(ptr(o));
      int64_t n = P.T[o].numel;
      const int* sd = reinterpret_cast<const int*>(ptr(O["seed"].i32()));
      uint32_t salt = (uint32_t)(((uint64_t)O["salt"].i64() * 0x9E3779B1ull) & 0xFFFFFFFFull);
      add("randn", [=](cudaStream_t s) { launch_randn(op, n, sd, salt, s); });
      continue;
    }
    if (k == "conv2d" || k == "conv2d_input_grad" || k == "conv2d_weight_grad" || k == "max_pool_2d" ||
        k == "max_pool_2d_grad") {
      ConvDesc c{};
      c.sH = O["strideH"].i32(); c.sW = O["strideW"].i32(); c.pH = O["padH"].i32(); c.pW = O["padW"].i32();
      c.G = O.find("groups") ? O["groups"].i32() : 1;
      if (k == "conv2d") {
        int x = O["input"].i32(), w = O["weight"].i32();
        ensure_contig(x, "conv2d"); ensure_contig(w, "conv2d");
        auto& xs = P.T[x].shape; auto& ws = P.T[w].shape;
        c.B = (int)xs[0]; c.Cin = (int)xs[1]; c.H = (int)xs[2]; c.W = (int)xs[3];
        c.Cout = (int)ws[0]; c.kH = (int)ws[2]; c.kW = (int)ws[3]; c.Hout = (int)os[2]; c.Wout = (int)os[3];
        const float* xp = (const float*)ptr(x); const float* wp = (const float*)ptr(w); float* yp = (float*)ptr(o);
        float* sc = (float*)scratch; int64_t sf = (int64_t)scratch_floats;
        emit_conv(0, c, xp, wp, yp, sc, sf, add);
      } else if (k == "conv2d_input_grad") {
        int w = O["weight"].i32(), dy = O["dy"].i32();
        ensure_contig(w, k.c_str()); ensure_contig(dy, k.c_str());
        auto& ws = P.T[w].shape; auto& ds = P.T[dy].shape;
        c.B = (int)os[0]; c.Cin = (int)os[1]; c.H = (int)os[2]; c.W = (int)os[3];
        c.Cout = (int)ws[0]; c.kH = (int)ws[2]; c.kW = (int)ws[3]; c.Hout = (int)ds[2]; c.Wout = (int)ds[3];
        const float* wp = (const float*)ptr(w); const float* dp2 = (const float*)ptr(dy); float* xp = (float*)ptr(o);
        float* sc = (float*)scratch; int64_t sf = (int64_t)scratch_floats;
        emit_conv(1, c, wp, dp2, xp, sc, sf, add);
      } else if (k == "conv2d_weight_grad") {
        int x = O["input"].i32(), dy = O["dy"].i32();
        ensure_contig(x, k.c_str()); ensure_contig(dy, k.c_str());
        auto& xs = P.T[x].shape; auto& ds = P.T[dy].shape;
        c.B = (int)xs[0]; c.Cin = (int)xs[1]; c.H = (int)xs[2]; c.W = (int)xs[3];
        c.Cout = (int)os[0]; c.kH = (int)os[2]; c.kW = (int)os[3]; c.Hout = (int)ds[2]; c.Wout = (int)ds[3];
        const float* xp = (const float*)ptr(x); const float* dp2 = (const float*)ptr(dy); float* wp = (float*)ptr(o);
        float* sc = (float*)scratch; int64_t sf = (int64_t)scratch_floats;
        emit_conv(2, c, xp, dp2, wp, sc, sf, add);
      } else {
        int x = O["input"].i32();
        ensure_contig(x, k.c_str());
        auto& xs = P.T[x].shape;
        c.B = (int)xs[0]; c.Cin = (int)xs[1]; c.H = (int)xs[2]; c.W = (int)xs[3];
        c.kH = O["kH"].i32(); c.kW = O["kW"].i32(); c.G = 1;
        const float* xp = (const float*)ptr(x);
        if (k == "max_pool_2d") {
          c.Hout = (int)os[2]; c.Wout = (int)os[3];
          float* yp = (float*)ptr(o);
          add(k, [=](cudaStream_t s) { launch_maxpool(c, xp, yp, s); });
        } else {
          int dy = O["dy"].i32();
          ensure_contig(dy, k.c_str());
          c.Hout = (int)P.T[dy].shape[2]; c.Wout = (int)P.T[dy].shape[3];
          const float* dp2 = (const float*)ptr(dy);
          float* dx = (float*)ptr(o);
          add(k, [=](cudaStream_t s) { launch_maxpool_grad(c, xp, dp2, dx, s); });
        }
      }
      continue;
    }
    throw TgError("Error", "no CUDA lowering for op kind '" + k + "'");
  }

  // Fused optimizer over the flat arenas.
  const float gscale = ctx->world > 1 ? 1.0f / (float)ctx->world : 1.0f;
  if (adam_fused_) {
    AdamFlatDesc d = adam_;
    d.p = reinterpret_cast<float*>(arena_[AR_PARAM]);
    d.g = reinterpret_cast<const float*>(arena_[AR_GRAD]);
    d.m = reinterpret_cast<float*>(arena_[AR_M]);
    d.v = reinterpret_cast<float*>(arena_[AR_V]);
    d.n = flat_floats_;
    d.n_decay = n_decay_;
    d.lrt = reinterpret_cast<const float*>(ptr(adam_lrt_));
    d.shrink_dev = adam_shrink_ >= 0 ? reinterpret_cast<const float*>(ptr(adam_shrink_)) : nullptr;
    d.grad_scale = gscale;
    next_bytes_ = 28.0 * (double)flat_floats_;  // read p, g, m, v; write p, m, v
    add("adam_flat", [d](cudaStream_t s) { launch_adam_flat(d, s); });
  } else if (sgd_fused_) {
    SgdFlatDesc d = sgd_;
    d.p = reinterpret_cast<float*>(arena_[AR_PARAM]);
    d.g = reinterpret_cast<const float*>(arena_[AR_GRAD]);
    d.v = sgd_.momentum > 0 ? reinterpret_cast<float*>(arena_[AR_M]) : nullptr;
    d.n = flat_floats_;
    d.n_decay = n_decay_;
    d.lr = reinterpret_cast<const float*>(ptr(sgd_lr_));
    d.grad_scale = gscale;
    next_bytes_ = (sgd_.momentum > 0 ? 20.0 : 12.0) * (double)flat_floats_;
    add("sgd_flat", [d](cudaStream_t s) { launch_sgd_flat(d, s); });
  } else {
    // Unfused optimizer graph: copy each new value to its home after all ops.
    for (auto& w : P.writebacks) {
      int src = w.src;
      int dst_t = -1;
      if (w.to_param) { for (auto& p : P.params) if (p.first == w.dest) dst_t = p.second; }
      else { for (auto& s2 : P.states) if (s2.name == w.dest) dst_t = s2.tensor; }
      if (dst_t < 0) throw TgError("Error", "writeback destination '" + w.dest + "' not found");
      void* dp2 = ptr(dst_t);
      const void* sp = ptr(src);
      size_t bytes = (size_t)P.T[src].numel * 4;
      add("writeback", [=](cudaStream_t s) { cudaMemcpyAsync(dp2, sp, bytes, cudaMemcpyDeviceToDevice, s); });
    }
  }
  if (ctx->world > 1 && !parent && P.loss >= 0) {
    float* la = reinterpret_cast<float*>(reinterpret_cast<char*>(arena_[AR_PERSIST]) + loss_avg_off_);
    const float* lp = reinterpret_cast<const float*>(ptr(P.loss));
    Context* c = ctx;
    float inv = 1.0f / (float)ctx->world;
    add("loss_allreduce", [=](cudaStream_t s) {
      cudaMemcpyAsync(la, lp, 4, cudaMemcpyDeviceToDevice, s);
      c->allreduce_sum(la, 1, s);
      launch_scale(la, 1, inv, s);
    });
  }
  if (!ctx->dry) jit_compile_pending();
}

// ------------------------------------------------------------ execution --
void Graph::run_launches(cudaStream_t s) {
  for (size_t i = 0; i < launches_.size(); ++i) {
    launches_[i](s);
    if (!captured_ && !use_graph_) {
      cudaError_t e = cudaGetLastError();
      if (e != cudaSuccess)
        throw TgError("CudaError", "launch '" + launch_kind_[i] + "': " + cudaGetErrorString(e));
    }
  }
}

void Graph::host_scalars() {
  cudaStream_t s = ctx->stream;
  auto put_f = [&](const std::string& name, float v) {
    auto it = P.inputs.find(name);
    if (it == P.inputs.end()) return;
    scalar_host_[scalar_n_] = v;
    TG_CUDA(cudaMemcpyAsync(ptr(it->second), &scalar_host_[scalar_n_], 4, cudaMemcpyHostToDevice, s));
    scalar_n_ = (scalar_n_ + 1) % (int)(sizeof(scalar_host_) / sizeof(float));
  };
  if (P.optimizer && !parent) {
    const auto& cfg = (*P.optimizer)["config"];
    const tgjson::Value& sched = has_lr_override_ ? lr_override_ : cfg["lr"];
    t_ += 1;
    double lr_now = resolve_lr(sched, t_);
    if ((*P.optimizer)["kind"].str() == "adam") {
      double b1 = cfg["beta1"].num(), b2 = cfg["beta2"].num();
      double lrt = lr_now * std::sqrt(1 - std::pow(b2, (double)t_)) / (1 - std::pow(b1, (double)t_));
      put_f(cfg["lrtInputName"].str(), (float)lrt);
      if (auto* dn = cfg.find("decayShrinkInputName"))
        if (!dn->is_null()) put_f(dn->str(), (float)(1 - lr_now * cfg["weightDecay"].num()));
    } else {
      put_f(cfg["lrInputName"].str(), (float)lr_now);
    }
  }
  if (P.uses_prng) {
    auto it = P.inputs.find("__prngSeed");
    if (it != P.inputs.end()) {
      prng_ += 1;
      int32_t v = (int32_t)prng_;
      float f;
      memcpy(&f, &v, 4);
      scalar_host_[scalar_n_] = f;
      TG_CUDA(cudaMemcpyAsync(ptr(it->second), &scalar_host_[scalar_n_], 4, cudaMemcpyHostToDevice, s));
      scalar_n_ = (scalar_n_ + 1) % (int)(sizeof(scalar_host_) / sizeof(float));
    }
  }
}

void Graph::launch_step() {
  cudaStream_t s = ctx->stream;
  ctx->check_comm();
  host_scalars();
  if (use_graph_) {
    if (!captured_) {
      TG_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
      try {
        run_launches(s);
      } catch (...) {
        cudaGraph_t g2 = nullptr;
        cudaStreamEndCapture(s, &g2);
        if (g2) cudaGraphDestroy(g2);
        throw;
      }
      TG_CUDA(cudaStreamEndCapture(s, &cgraph_));
      TG_CUDA(cudaGraphInstantiate(&cexec_, cgraph_, 0));
      captured_ = true;
    }
    TG_CUDA(cudaGraphLaunch(cexec_, s));
  } else {
    run_launches(s);
  }
}

void Graph::read_loss(float* out) {
  cudaStream_t s = ctx->stream;
  const void* src = (ctx->world > 1 && !parent)
                        ? reinterpret_cast<char*>(arena_[AR_PERSIST]) + loss_avg_off_
                        : ptr(P.loss);
  TG_CUDA(cudaMemcpyAsync(loss_host_, src, 4, cudaMemcpyDeviceToHost, s));
  if (parent) TG_CUDA(cudaStreamSynchronize(s));
  else ctx->sync(s);
  TG_CUDA(cudaGetLastError());
  *out = loss_host_[0];
}

void Graph::read_output(void* out) {
  int t = P.outputs.at(0);
  TG_CUDA(cudaMemcpyAsync(out, ptr(t), (size_t)P.T[t].numel * 4, cudaMemcpyDeviceToHost, ctx->stream));
  TG_CUDA(cudaStreamSynchronize(ctx->stream));
}

void Graph::read_captures(void* const* out) {
  for (size_t i = 0; i < P.captures.size(); ++i) {
    if (!out[i]) continue;
    int t = P.captures[i].second;
    TG_CUDA(cudaMemcpyAsync(out[i], ptr(t), (size_t)P.T[t].numel * 4, cudaMemcpyDeviceToHost, ctx->stream));
  }
  TG_CUDA(cudaStreamSynchronize(ctx->stream));
}

void Graph::read_tensor(int t, void* out) {
  if (t < 0 || t >= (int)P.T.size()) throw TgError("Error", "tensor id out of range");
  if (views_[t].onehot || loc_[views_[t].root].arena == -1)
    throw TgError("Error", "tensor #" + std::to_string(t) + " has no persistent storage");
  int ar = loc_[views_[t].root].arena;
  if (ar == AR_TEMP || !views_[t].contiguous)
    throw TgError("Error", "tensor #" + std::to_string(t) + " is a pooled temporary");
  TG_CUDA(cudaMemcpyAsync(out, ptr(t), (size_t)P.T[t].numel * 4, cudaMemcpyDeviceToHost, ctx->stream));
  TG_CUDA(cudaStreamSynchronize(ctx->stream));
}

void Graph::read_grad(const std::string& name, float* out) {
  auto it = param_off_.find(name);
  if (it == param_off_.end() || !arena_[AR_GRAD]) throw TgError("Error", "no gradient for '" + name + "'");
  TG_CUDA(cudaMemcpyAsync(out, reinterpret_cast<char*>(arena_[AR_GRAD]) + it->second,
                          (size_t)param_n_[name] * 4, cudaMemcpyDeviceToHost, ctx->stream));
  TG_CUDA(cudaStreamSynchronize(ctx->stream));
}

// Every declared input except those the runtime writes itself (the PRNG
// seed and the optimizer's per-step scalars) must come with a step or a run
// (src/runtime.ts:322-328).
void Graph::require_inputs(int n, const char* const* names) const {
  std::set<std::string> given(names, names + n), injected{"__prngSeed"};
  if (P.optimizer) {
    const auto& cfg = (*P.optimizer)["config"];
    for (const char* k : {"lrtInputName", "decayShrinkInputName", "lrInputName"})
      if (auto* v = cfg.find(k))
        if (!v->is_null()) injected.insert(v->str());
  }
  for (const auto& kv : P.inputs)
    if (!injected.count(kv.first) && !given.count(kv.first))
      throw TgError("Error", "missing input '" + kv.first + "'");
}

void Graph::set_inputs(int n, const char* const* names, const void* const* data, const size_t* bytes,
                       bool device_src) {
  for (int i = 0; i < n; ++i) {
    auto it = P.inputs.find(names[i]);
    if (it == P.inputs.end()) throw TgError("Error", std::string("unknown input '") + names[i] + "'");
    int t = it->second;
    size_t want = (size_t)P.T[t].numel * 4;
    if (bytes[i] != want)
      throw TgError("Error", std::string("input '") + names[i] + "' has " + std::to_string(bytes[i]) +
                                 " bytes, expected " + std::to_string(want));
    TG_CUDA(cudaMemcpyAsync(ptr(t), data[i], want, device_src ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                            ctx->stream));
  }
}

void Graph::upload_params(int n, const char* const* names, const float* const* data, const size_t* numel) {
  for (int i = 0; i < n; ++i) {
    float* p = param_ptr(names[i]);
    if (!p) throw TgError("Error", std::string("uploadParams: unknown param '") + names[i] + "'");
    if ((int64_t)numel[i] != param_numel(names[i]))
      throw TgError("Error", std::string("uploadParams: size mismatch for '") + names[i] + "'");
    TG_CUDA(cudaMemcpyAsync(p, data[i], numel[i] * 4, cudaMemcpyHostToDevice, ctx->stream));
  }
  TG_CUDA(cudaStreamSynchronize(ctx->stream));
}

void Graph::download_params(int n, const char* const* names, float* const* out, const size_t* numel) {
  for (int i = 0; i < n; ++i) {
    float* p = param_ptr(names[i]);
    if (!p) throw TgError("Error", std::string("downloadParams: unknown param '") + names[i] + "'");
    if ((int64_t)numel[i] != param_numel(names[i]))
      throw TgError("Error", std::string("downloadParams: size mismatch for '") + names[i] + "'");
    TG_CUDA(cudaMemcpyAsync(out[i], p, numel[i] * 4, cudaMemcpyDeviceToHost, ctx->stream));
  }
  TG_CUDA(cudaStreamSynchronize(ctx->stream));
}

// Optimizer state by name (adam_m_<param>, adam_v_<param>, sgd_v_<param>, or
// any other state_input), for checkpoints.
int Graph::state_tensor(const std::string& name) const {
  for (auto& st : P.states)
    if (st.name == name) return st.tensor;
  return -1;
}

void Graph::upload_states(int n, const char* const* names, const float* const* data, const size_t* numel) {
  for (int i = 0; i < n; ++i) {
    const int t = state_tensor(names[i]);
    if (t < 0 || loc_[views_[t].root].arena < 0)
      throw TgError("Error", std::string("uploadState: unknown state '") + names[i] + "'");
    if ((int64_t)numel[i] != P.T[t].numel)
      throw TgError("Error", std::string("uploadState: size mismatch for '") + names[i] + "'");
    TG_CUDA(cudaMemcpyAsync(ptr(t), data[i], numel[i] * 4, cudaMemcpyHostToDevice, ctx->stream));
  }
  TG_CUDA(cudaStreamSynchronize(ctx->stream));
}

void Graph::download_states(int n, const char* const* names, float* const* out, const size_t* numel) {
  for (int i = 0; i < n; ++i) {
    const int t = state_tensor(names[i]);
    if (t < 0 || loc_[views_[t].root].arena < 0)
      throw TgError("Error", std::string("downloadState: unknown state '") + names[i] + "'");
    if ((int64_t)numel[i] != P.T[t].numel)
      throw TgError("Error", std::string("downloadState: size mismatch for '") + names[i] + "'");
    TG_CUDA(cudaMemcpyAsync(out[i], ptr(t), numel[i] * 4, cudaMemcpyDeviceToHost, ctx->stream));
  }
  TG_CUDA(cudaStreamSynchronize(ctx->stream));
}

void Graph::reset_optimizer() {
  cudaStream_t s = ctx->stream;
  for (int a : {AR_M, AR_V}) if (arena_[a]) TG_CUDA(cudaMemsetAsync(arena_[a], 0, (size_t)arena_bytes_[a], s));
  for (auto& st : P.states) {
    int t = st.tensor;
    if (loc_[t].arena < 0) continue;
    float v = (float)st.init;
    uint32_t bits;
    memcpy(&bits, &v, 4);
    launch_fill(ptr(t), P.T[t].numel, bits, s);
  }
  t_ = 0;
  TG_CUDA(cudaStreamSynchronize(s));
}

void Graph::set_lr(const char* lr_json, size_t len) {
  lr_override_ = tgjson::parse(lr_json, len);
  has_lr_override_ = true;
}

void Graph::profile_step(std::vector<float>& ms) {
  cudaStream_t s = ctx->stream;
  host_scalars();
  std::vector<cudaEvent_t> ev(launches_.size() + 1);
  for (auto& x : ev) TG_CUDA(cudaEventCreate(&x));
  // The launches and an event record node after each run as one CUDA graph,
  // as the step itself does, so each interval is the kernel plus the graph's
  // own node-to-node latency rather than the host's launch rate.
  bool graphed = false;
  if (use_graph_ && cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
    cudaGraph_t g = nullptr;
    cudaGraphExec_t gx = nullptr;
    bool ok = cudaEventRecordWithFlags(ev[0], s, cudaEventRecordExternal) == cudaSuccess;
    try {
      for (size_t i = 0; ok && i < launches_.size(); ++i) {
        launches_[i](s);
        ok = cudaEventRecordWithFlags(ev[i + 1], s, cudaEventRecordExternal) == cudaSuccess;
      }
    } catch (...) {
      ok = false;
    }
    ok = cudaStreamEndCapture(s, &g) == cudaSuccess && ok;
    if (ok && cudaGraphInstantiate(&gx, g, 0) == cudaSuccess) {
      graphed = cudaGraphLaunch(gx, s) == cudaSuccess;
      TG_CUDA(cudaStreamSynchronize(s));
      cudaGraphExecDestroy(gx);
    }
    if (g) cudaGraphDestroy(g);
    cudaGetLastError();
  }
  if (!graphed) {
    // eager fallback: the GPU waits while the host enqueues every launch and
    // event, so the events time the kernels back to back
    const uint64_t hold_ns =
        std::min<uint64_t>(200000000ull, std::max<uint64_t>(5000000ull, 20000ull * launches_.size()));
    launch_gpu_delay(hold_ns, s);
    TG_CUDA(cudaEventRecord(ev[0], s));
    for (size_t i = 0; i < launches_.size(); ++i) {
      launches_[i](s);
      TG_CUDA(cudaEventRecord(ev[i + 1], s));
    }
  }
  TG_CUDA(cudaStreamSynchronize(s));
  TG_CUDA(cudaGetLastError());
  ms.assign(launches_.size(), 0.f);
  for (size_t i = 0; i < launches_.size(); ++i) TG_CUDA(cudaEventElapsedTime(&ms[i], ev[i], ev[i + 1]));
  for (auto& x : ev) cudaEventDestroy(x);
}

std::string Graph::launch_kinds() const {
  std::string s;
  for (auto& k : launch_kind_) { s += k; s += '\n'; }
  return s;
}

std::string Graph::info_json() const {
  std::string s = "{\"params\":[";
  for (size_t i = 0; i < P.params.size(); ++i) {
    if (i) s += ",";
    s += "\"" + P.params[i].first + "\"";
  }
  s += "],\"launches\":" + std::to_string(launches_.size());
  s += ",\"fusedOptimizer\":" + std::string(adam_fused_ ? "\"adam\"" : sgd_fused_ ? "\"sgd\"" : "null");
  int64_t total = 0;
  for (int a = 0; a < AR_COUNT; ++a) if (arena_owned_[a]) total += arena_bytes_[a];
  s += ",\"deviceBytes\":" + std::to_string(total);
  s += ",\"tempBytes\":" + std::to_string(arena_bytes_[AR_TEMP]);
  s += ",\"flatFloats\":" + std::to_string(flat_floats_);
  s += "}";
  return s;
}

// ---------------------------------------------------------------- Context --
// Collective failure handling (data parallel only).
//
// TG_NCCL_TIMEOUT_S (default 300) bounds communicator set-up and every step's
// completion wait. TG_FAULT injects failures on the host, faking the result
// of the call that fails rather than breaking anything on the GPU:
//   nccl_init        communicator set-up reports an error;
//   nccl_init_stall  set-up never completes (the deadline and abort path runs);
//   step_error:N     the N-th step's completion check reports an NCCL error;
//   step_stall:N     the N-th step's completion is never observed (deadline).
// The first two act before any CUDA call, so they also run on machines
// without a GPU.
static double nccl_timeout_s() {
  const char* e = getenv("TG_NCCL_TIMEOUT_S");
  const double v = e ? atof(e) : 300.0;
  return v > 0 ? v : 300.0;
}
static std::string tg_fault() {
  const char* e = getenv("TG_FAULT");
  return e ? std::string(e) : std::string();
}
// The step number N of a "name:N" fault, or -1.
static int64_t fault_step(const std::string& f, const char* name) {
  const std::string p = std::string(name) + ":";
  return f.rfind(p, 0) == 0 ? atoll(f.c_str() + p.size()) : -1;
}
// Polls until poll() returns 0 (done) or -1 (failed), or the deadline passes;
// returns 0, -1, or 1 (timed out).
template <class Poll>
static int poll_until(double timeout_s, Poll poll) {
  const auto t0 = std::chrono::steady_clock::now();
  for (int it = 0;; ++it) {
    const int r = poll();
    if (r <= 0) return r;
    if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > timeout_s) return 1;
    std::this_thread::sleep_for(std::chrono::microseconds(it < 64 ? 2 : 50));
  }
}

Context::Context(int dev, int rk, int wd, const unsigned char* nccl_id) : device(dev), rank(rk), world(wd) {
  const std::string fault = world > 1 ? tg_fault() : std::string();
  if (fault == "nccl_init")
    throw TgError("NcclError", "ncclCommInitRankConfig: injected failure (TG_FAULT=nccl_init)");
  if (fault == "nccl_init_stall") {
    const double to = nccl_timeout_s();
    poll_until(to, [] { return 1; });  // set-up that never completes
    throw TgError("NcclError", "communicator set-up did not complete within " + std::to_string(to) +
                                   " s (TG_FAULT=nccl_init_stall); communicator aborted");
  }
  TG_CUDA(cudaSetDevice(dev));
  TG_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
  if (world > 1) {
    if (!nccl_id) throw TgError("NcclError", "world > 1 needs an NCCL unique id");
    ncclUniqueId id;
    memcpy(&id, nccl_id, sizeof(id));
    ncclComm_t comm = nullptr;
    // Non-blocking set-up, polled against the deadline: a peer that never
    // joins ends in ncclCommAbort and an NcclError instead of a hang.
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclResult_t r = ncclCommInitRankConfig(&comm, world, id, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress)
      throw TgError("NcclError", std::string("ncclCommInitRankConfig: ") + ncclGetErrorString(r));
    ncclResult_t st = ncclInProgress;
    const double to = nccl_timeout_s();
    const int w = poll_until(to, [&] {
      if (ncclCommGetAsyncError(comm, &st) != ncclSuccess) return -1;
      return st == ncclInProgress ? 1 : (st == ncclSuccess ? 0 : -1);
    });
    if (w != 0) {
      ncclCommAbort(comm);
      throw TgError("NcclError", w > 0 ? "communicator set-up did not complete within " + std::to_string(to) +
                                             " s (a peer rank never joined); communicator aborted"
                                       : std::string("communicator set-up failed: ") + ncclGetErrorString(st));
    }
    nccl = comm;
    int lo = 0, hi = 0;
    TG_CUDA(cudaDeviceGetStreamPriorityRange(&lo, &hi));
    TG_CUDA(cudaStreamCreateWithPriority(&comm_stream, cudaStreamNonBlocking, hi));
  }
}

Context::Context(Dry, int wd) : device(-1), rank(0), world(wd), dry(true) {}

Context::~Context() {
  graphs.clear();
  if (nccl && !nccl_aborted) ncclCommDestroy(reinterpret_cast<ncclComm_t>(nccl));
  if (comm_stream) cudaStreamDestroy(comm_stream);
  if (stream) cudaStreamDestroy(stream);
}

// On a non-blocking communicator a call may return ncclInProgress; its
// enqueue is complete once ncclCommGetAsyncError stops reporting that, and
// the next NCCL call (or the end of a stream capture) must wait for it.
static ncclResult_t settle(ncclComm_t comm, ncclResult_t r) {
  if (r != ncclInProgress) return r;
  ncclResult_t st = ncclInProgress;
  const int w = poll_until(nccl_timeout_s(), [&] {
    if (ncclCommGetAsyncError(comm, &st) != ncclSuccess) return -1;
    return st == ncclInProgress ? 1 : 0;
  });
  return w == 0 ? st : ncclInternalError;
}

void Context::check_comm() const {
  if (nccl_aborted) throw TgError("NcclError", "the communicator was aborted after an earlier collective failure");
}

void Context::allreduce_ranges(const std::vector<std::pair<float*, int64_t>>& ranges, cudaStream_t s) {
  check_comm();
  ncclComm_t comm = reinterpret_cast<ncclComm_t>(nccl);
  ncclResult_t r = settle(comm, ncclGroupStart());
  for (size_t i = 0; r == ncclSuccess && i < ranges.size(); ++i)
    r = settle(comm, ncclAllReduce(ranges[i].first, ranges[i].first, (size_t)ranges[i].second, ncclFloat32, ncclSum,
                                   comm, s));
  const ncclResult_t r2 = settle(comm, ncclGroupEnd());
  if (r != ncclSuccess || r2 != ncclSuccess)
    throw TgError("NcclError", std::string("ncclAllReduce (bucket): ") + ncclGetErrorString(r != ncclSuccess ? r : r2));
}

void Context::allreduce_sum(float* buf, int64_t n, cudaStream_t s) {
  check_comm();
  ncclComm_t comm = reinterpret_cast<ncclComm_t>(nccl);
  ncclResult_t r = settle(comm, ncclAllReduce(buf, buf, (size_t)n, ncclFloat32, ncclSum, comm, s));
  if (r != ncclSuccess) throw TgError("NcclError", std::string("ncclAllReduce: ") + ncclGetErrorString(r));
}

// ncclCommAbort on a detached host thread, waited for at most timeout_s,
// then a bounded wait for the stream: on this pool an abort issued by both
// ranks of a communicator at once was seen not to return (NCCL 2.28.9), and a
// failing step must still come back to its caller with an error.
static void abort_bounded(ncclComm_t comm, cudaStream_t s, double timeout_s) {
  auto done = std::make_shared<std::atomic<bool>>(false);
  std::thread([comm, done] {
    ncclCommAbort(comm);
    done->store(true);
  }).detach();
  poll_until(timeout_s, [&] { return done->load() ? 0 : 1; });
  poll_until(timeout_s, [&] {
    const cudaError_t e = cudaStreamQuery(s);
    return e == cudaErrorNotReady ? 1 : 0;
  });
}

void Context::sync(cudaStream_t s) {
  if (!nccl) {
    TG_CUDA(cudaStreamSynchronize(s));
    return;
  }
  check_comm();
  const int64_t n = ++dp_syncs;
  const std::string fault = tg_fault();
  const bool stall = fault_step(fault, "step_stall") == n, err = fault_step(fault, "step_error") == n;
  ncclComm_t comm = reinterpret_cast<ncclComm_t>(nccl);
  cudaError_t ce = cudaSuccess;
  ncclResult_t st = ncclSuccess;
  const double to = nccl_timeout_s();
  const int w = poll_until(to, [&] {
    ce = cudaStreamQuery(s);
    if (ce != cudaSuccess && ce != cudaErrorNotReady) return -1;
    if (ncclCommGetAsyncError(comm, &st) != ncclSuccess || (st != ncclSuccess && st != ncclInProgress)) {
      ce = cudaSuccess;
      return -1;
    }
    if (ce != cudaSuccess) return 1;  // still running
    // injected faults are reported only once the step's work has finished on
    // this device, so the abort below never cuts a collective short
    if (err) { st = ncclRemoteError; return -1; }
    return stall ? 1 : 0;
  });
  if (w == 0) return;
  if (ce != cudaSuccess) throw TgError("CudaError", std::string("step: ") + cudaGetErrorString(ce));
  if (w > 0) {
    // the step's work may still be queued behind a collective that waits on
    // a peer: abort it, then wait for the stream to drain
    if (!nccl_aborted) abort_bounded(comm, s, to);
    nccl_aborted = true;
    throw TgError("NcclError", "step did not complete within " + std::to_string(to) + " s" +
                                   (stall ? " (TG_FAULT=step_stall)" : " (a peer rank stalled or left)") +
                                   "; communicator aborted");
  }
  if (!nccl_aborted) abort_bounded(comm, s, to);
  nccl_aborted = true;
  throw TgError("NcclError", std::string("collective failed: ") + ncclGetErrorString(st) +
                                 (err ? " (TG_FAULT=step_error)" : "") + "; communicator aborted");
}

}  // namespace tg
