// Elementwise fusion: groups of elementwise IR ops become one generated
// kernel each.
//
// The reference runs every IR op as its own WGSL kernel and stores every
// intermediate (src/codegen.ts:107-330, one shader per op). On B200 those
// ops are HBM-bound, so a chain such as GELU's seven ops re-reads and
// re-writes the activation seven times. Here an elementwise op absorbs the
// elementwise ops that produce its operands when the produced tensor
//   * has exactly one consumer (this op) and no view of it is taken,
//   * is not observable from the host (loss, output, capture, gradient,
//     writeback source),
//   * has the consumer's output shape, or broadcasts to it and contains no
//     position-dependent op (its value is then recomputed per element), and
//   * sits on the same side of the optimizer section.
// The absorbed tensors get no storage. Each group is written out as CUDA C
// with shapes, strides and constants as literals (dims divide by constants,
// broadcasts become index arithmetic the compiler folds), compiled by NVRTC
// (jit.cu) and launched as one grid-stride kernel, 4 elements per thread with
// 128-bit loads and stores whenever every operand allows it.
//
// Every op's arithmetic is the same f32 operation, rounded the same way, as
// the unfused interpreter kernel (kernels_ew.cu) performs for it, so fusion
// changes which values reach HBM, not the values.
#include <algorithm>
#include <cstring>
#include <functional>
#include <set>
#include <sstream>

#include "runtime.hpp"

namespace tg {

namespace {

bool jit_enabled() {
  const char* e = getenv("TG_EW_JIT");
  return !(e && e[0] == '0');
}

}  // namespace

const std::set<std::string>& ew_kinds() {
  static const std::set<std::string> s = {
      "add", "sub", "mul", "div", "min", "max", "less", "greater",
      "sqrt", "rsqrt", "log", "exp", "relu", "neg", "abs", "tanh", "sigmoid", "erf", "sin", "cos",
      "mul_scalar", "add_scalar", "where_causal", "dropout", "broadcast_to", "where", "relu_grad",
      "adam_update_m", "adam_update_v", "adam_update_p"};
  return s;
}

// Operand tensors of an elementwise op, in the order its expression reads them.
std::vector<int> ew_operands(const Program& P, int i) {
  const std::string& k = P.kind[i];
  const auto& O = P.op(i);
  if (k == "where") return {O["cond"].i32(), O["a"].i32(), O["b"].i32()};
  if (k == "relu_grad") return {O["x"].i32(), O["dy"].i32()};
  if (k == "adam_update_m") return {O["m"].i32(), O["g"].i32()};
  if (k == "adam_update_v") return {O["v"].i32(), O["g"].i32()};
  if (k == "adam_update_p") {
    std::vector<int> v = {O["p"].i32(), O["mNew"].i32(), O["lrt"].i32()};
    if (!O["decayShrinkTensor"].is_null()) v.push_back(O["decayShrinkTensor"].i32());
    v.push_back(O["vNew"].i32());
    return v;
  }
  static const std::set<std::string> binary = {"add", "sub", "mul", "div", "min", "max", "less", "greater"};
  if (binary.count(k)) return {O["a"].i32(), O["b"].i32()};
  return {O["a"].i32()};
}

namespace {

// Exact f32 literal in generated source.
std::string lit(float f) {
  uint32_t b;
  memcpy(&b, &f, 4);
  char buf[32];
  snprintf(buf, sizeof buf, "tg_bits(0x%08xu)", b);
  return buf;
}

// Right-aligned broadcast of shape a onto shape b.
bool broadcasts_to(const std::vector<int64_t>& a, const std::vector<int64_t>& b) {
  if (a.size() > b.size()) return false;
  const size_t off = b.size() - a.size();
  for (size_t d = 0; d < a.size(); ++d)
    if (a[d] != 1 && a[d] != b[off + d]) return false;
  return true;
}

// Ops that cost tens of instructions per element (SFU sequences, IEEE
// division): worth computing once per value rather than once per broadcast
// element.
bool expensive_kind(const std::string& k) {
  return k == "sqrt" || k == "rsqrt" || k == "div" || k == "exp" || k == "log" || k == "tanh" ||
         k == "sigmoid" || k == "erf" || k == "sin" || k == "cos";
}

constexpr int kMaxGroupInputs = 12;
constexpr int kMaxGroupOps = 48;

}  // namespace

// A row reduction's per-row values (its result and its post ops' results),
// each mapped to itself, plus the reshapes / stop_gradients of them that keep
// the element count (keepDims adds a unit dimension), each mapped to the value
// it aliases.
std::map<int, int> Graph::row_values(const EwGroup& G) const {
  std::map<int, int> rv = {{P.out[G.red], P.out[G.red]}};
  for (int pr : G.post_roots) rv[P.out[pr]] = P.out[pr];
  std::vector<int> work;
  for (const auto& kv : rv) work.push_back(kv.first);
  while (!work.empty()) {
    const int x = work.back();
    work.pop_back();
    for (int c : P.consumers[x]) {
      const int y = P.out[c];
      if ((P.kind[c] == "reshape" || P.kind[c] == "stop_gradient") && P.T[y].numel == P.T[x].numel && !rv.count(y)) {
        rv[y] = rv[x];
        work.push_back(y);
      }
    }
  }
  return rv;
}

// The tensors that alias value t through element-count-preserving reshapes
// and stop_gradients (views), t included.
static std::set<int> view_aliases(const Program& P, int t) {
  std::set<int> s = {t};
  std::vector<int> work = {t};
  while (!work.empty()) {
    const int x = work.back();
    work.pop_back();
    for (int c : P.consumers[x])
      if ((P.kind[c] == "reshape" || P.kind[c] == "stop_gradient") && P.T[P.out[c]].numel == P.T[x].numel &&
          s.insert(P.out[c]).second)
        work.push_back(P.out[c]);
  }
  return s;
}

// True when an elementwise group over shape vshape (rows of length len)
// reads tensor x as one value per row: element (r, j) of the group takes
// element r of x. A per-row value reshaped so that it broadcasts another way
// (a [1, N] or [N] view of an [N, 1] row result over [N, N]) is not.
bool Graph::reads_as_row(int x, const std::vector<int64_t>& vshape, int64_t len) {
  bool dummy = true;
  const EwInput in = ew_input(x, vshape, dummy, false);
  if (in.mode == IN_ROWDIV) return in.period == len;
  if (in.mode == IN_SCALAR) {
    int64_t n = 1;
    for (int64_t d : vshape) n *= d;
    return n == len;  // a single row
  }
  return false;
}

bool Graph::ew_internal(int t) const {
  if (ew_absorbed_.empty()) return false;
  const int p = P.producer[t];
  return p >= 0 && ew_absorbed_[p] && !ew_post_[p];
}

namespace {
// How a reduction consumes its input: along the last axis (rows) or the
// leading axes (columns), or neither (not fused).
enum RedShape { RED_NONE = 0, RED_ROW, RED_COL };
// Rows up to this length are reduced by one warp each (and may carry post
// ops and an epilogue); longer rows by one 256-thread block each.
constexpr int64_t kWarpRowMax = 4096;
RedShape red_shape(const Program& P, int r, int64_t* rows, int64_t* len) {
  const std::string& k = P.kind[r];
  if (k != "sum_last" && k != "mean_last" && k != "sum_to_shape") return RED_NONE;
  const int a = P.op(r)["a"].i32();
  const auto& is = P.T[a].shape;
  const int64_t n = P.T[a].numel, on = P.T[P.out[r]].numel;
  if (n <= 0 || on <= 0) return RED_NONE;
  if (k == "sum_last" || k == "mean_last") {
    *len = is.empty() ? 1 : is.back();
    *rows = n / std::max<int64_t>(*len, 1);
    return RED_ROW;
  }
  if (k != "sum_to_shape") return RED_NONE;
  const auto& os = P.T[P.out[r]].shape;
  const int R = (int)is.size(), rd = R - (int)os.size();
  std::vector<int> keep(R, 0);
  for (int d = 0; d < R; ++d) keep[d] = (d >= rd && !(os[d - rd] == 1 && is[d] != 1)) ? 1 : 0;
  bool prefix = true, suffix = true, seen_red = false, seen_keep = false;
  for (int d = 0; d < R; ++d) {
    if (is[d] == 1) continue;
    if (!keep[d]) { seen_red = true; if (seen_keep) suffix = false; }
    else { seen_keep = true; if (seen_red) prefix = false; }
  }
  if (on == n) return RED_NONE;  // nothing reduced (a view or a copy)
  if (prefix && !suffix) { *rows = on; *len = n / on; return RED_ROW; }
  if (suffix && !prefix) { *rows = n / on; *len = on; return RED_COL; }
  return RED_NONE;
}
}  // namespace

void Graph::plan_fusion() {
  const int nO = (int)P.ops.size();
  ew_group_.assign(nO, -1);
  ew_absorbed_.assign(nO, 0);
  ew_post_.assign(nO, 0);
  ew_groups_.clear();
  jit_ = jit_enabled();
  if (!jit_) return;
  std::set<int> observable;
  for (int t : P.outputs) observable.insert(t);
  for (auto& c : P.captures) observable.insert(c.second);
  for (auto& w : P.writebacks) observable.insert(w.src);
  for (auto& g : P.grads) observable.insert(g.second);
  if (P.loss >= 0) observable.insert(P.loss);
  auto is_ew = [&](int i) { return !op_done_[i] && action_[i] == 0 && ew_kinds().count(P.kind[i]) > 0; };
  auto side = [&](int i) { return P.opt_start >= 0 && i >= P.opt_start; };
  // A produced tensor a consumer may evaluate in place: its own storage, not
  // observable, and read at the consumer's shape or broadcast to it.
  auto inlinable = [&](int t) {
    const TView& v = views_[t];
    return !observable.count(t) && v.root == t && !v.onehot && v.contiguous;
  };

  // Working state per op that roots a group.
  std::vector<char> root(nO, 0), posdep(nO, 0);
  std::vector<std::vector<int>> mem(nO);
  std::vector<std::set<int>> ext(nO);  // tensors the group reads from memory
  std::vector<int> copied(P.T.size(), 0);  // consumers that evaluate the tensor in place
  auto full_inputs = [&](int p) {
    int n = 0;
    for (int t : ext[p]) if (P.T[t].numel >= P.T[P.out[p]].numel) ++n;
    return n;
  };
  auto merge_into = [&](int i, int p, int t) -> bool {
    std::set<int> merged = ext[i];
    merged.erase(t);
    merged.insert(ext[p].begin(), ext[p].end());
    std::vector<int> m = mem[i];
    m.insert(m.end(), mem[p].begin(), mem[p].end());
    std::sort(m.begin(), m.end());
    m.erase(std::unique(m.begin(), m.end()), m.end());
    if ((int)merged.size() > kMaxGroupInputs || (int)m.size() > kMaxGroupOps) return false;
    ext[i] = std::move(merged);
    mem[i] = std::move(m);
    posdep[i] = posdep[i] || posdep[p];
    return true;
  };

  for (int i = 0; i < nO; ++i) {
    if (!is_ew(i)) continue;
    root[i] = 1;
    mem[i] = {i};
    posdep[i] = P.kind[i] == "dropout" || P.kind[i] == "where_causal";
    for (int t : ew_operands(P, i)) ext[i].insert(t);
    std::set<int> seen;
    for (int t : ew_operands(P, i)) {
      if (!seen.insert(t).second) continue;
      const int p = P.producer[t];
      if (p < 0 || !root[p] || !inlinable(t) || side(p) != side(i)) continue;
      if (P.T[t].shape != P.T[P.out[i]].shape &&
          (!broadcasts_to(P.T[t].shape, P.T[P.out[i]].shape) || posdep[p]))
        continue;
      // a broadcast producer is recomputed for every element it is read at:
      // keep expensive row-level values (sqrt, division, ...) materialised
      if (P.T[t].numel * 8 <= P.T[P.out[i]].numel) {
        bool costly = false;
        for (int m : mem[p]) costly = costly || expensive_kind(P.kind[m]);
        if (costly) continue;
      }
      const std::vector<int> cs = eff_consumers(t);
      if (cs.size() == 1) {
        // sole consumer: the producer's group moves into this one
        if (merge_into(i, p, t)) { root[p] = 0; ext[p].clear(); }
        continue;
      }
      // Several elementwise consumers of a cheap group (at most one input as
      // large as its output, few ops): each consumer recomputes it rather than
      // reading it back; once all of them do, it is never stored.
      bool all_ew = true;
      for (int c : cs)
        if (!is_ew(c) || side(c) != side(p) ||
            !broadcasts_to(P.T[t].shape, P.T[P.out[c]].shape) ||
            (posdep[p] && P.T[t].shape != P.T[P.out[c]].shape))
          all_ew = false;
      if (!all_ew || full_inputs(p) > 1 || mem[p].size() > 16) continue;
      if (merge_into(i, p, t)) ++copied[t];
    }
  }
  // Producers whose every consumer evaluates them in place are not stored.
  for (int p = 0; p < nO; ++p)
    if (root[p] && copied[P.out[p]] > 0 && copied[P.out[p]] == (int)eff_consumers(P.out[p]).size()) root[p] = 0;

  // A reduction over the output of a group it alone consumes evaluates the
  // group per element instead of reading it back.
  std::vector<int> red_of(nO, -1);
  for (int r = 0; r < nO; ++r) {
    if (op_done_[r] || action_[r] != 0) continue;
    int64_t rows = 0, len = 0;
    if (red_shape(P, r, &rows, &len) == RED_NONE) continue;
    const int t = P.op(r)["a"].i32(), p = P.producer[t];
    if (p < 0 || !root[p] || !inlinable(t) || side(p) != side(r)) continue;
    if (eff_consumers(t).size() != 1 || (int)ext[p].size() > kMaxGroupInputs) continue;
    red_of[p] = r;
  }

  // Materialise the groups; every member not rooting one is absorbed.
  for (int i = 0; i < nO; ++i)
    if (is_ew(i) && !root[i]) ew_absorbed_[i] = 1;
  for (int p = 0; p < nO; ++p) {
    if (!root[p]) continue;
    EwGroup g;
    g.members = mem[p];
    if (red_of[p] >= 0) {
      ew_absorbed_[p] = 1;
      g.root = g.red = red_of[p];
    } else {
      g.root = p;
    }
    ew_group_[g.root] = (int)ew_groups_.size();
    ew_groups_.push_back(std::move(g));
  }

  // Post ops: a group with one value per row that reads a warp-per-row
  // reduction's result, and otherwise only per-row tensors produced earlier
  // or scalars, is evaluated by lane 0 of the reduction kernel after the sum
  // (LayerNorm's eps and sqrt on the variance, the row terms of its
  // gradient). Each such group saves a launch; the reduction's own result is
  // still written.
  std::map<int, std::vector<int>> owners;  // member op -> groups containing it
  for (size_t gi = 0; gi < ew_groups_.size(); ++gi)
    for (int m : ew_groups_[gi].members) owners[m].push_back((int)gi);
  for (size_t ri = 0; ri < ew_groups_.size(); ++ri) {
    EwGroup& R = ew_groups_[ri];
    if (R.red < 0) continue;
    int64_t rows = 0, len = 0;
    if (red_shape(P, R.red, &rows, &len) != RED_ROW || len > kWarpRowMax) continue;
    const int t = P.out[R.red];
    if (P.T[t].numel != rows || !views_[t].contiguous || views_[t].onehot) continue;
    std::set<int> post(R.post.begin(), R.post.end());
    for (int c : P.consumers[t]) {
      auto it = owners.find(c);
      if (it == owners.end()) continue;
      for (int ci : it->second) {
        EwGroup& C = ew_groups_[ci];
        if (ci == (int)ri || C.red >= 0 || C.root < 0 || ew_group_[C.root] != ci) continue;
        if (P.T[P.out[C.root]].numel != rows || side(C.root) != side(R.red)) continue;
        const std::set<int> cm(C.members.begin(), C.members.end());
        bool ok = (int)(post.size() + C.members.size()) <= kMaxGroupOps && R.post_roots.size() < 4;
        for (int m : C.members) {
          if (P.kind[m] == "dropout" || P.kind[m] == "where_causal") ok = false;
          if (P.T[P.out[m]].numel != rows) ok = false;
          for (int x : ew_operands(P, m)) {
            if (x == t || cm.count(P.producer[x])) continue;
            const TView& vx = views_[x];
            const bool stored =
                vx.contiguous && !vx.onehot && vx.root == x && !ew_internal(x) && P.producer[x] < R.red;
            if (!stored || (P.T[x].numel != 1 && P.T[x].numel != rows)) ok = false;
          }
        }
        if (!ok) continue;
        post.insert(C.members.begin(), C.members.end());
        R.post_roots.push_back(C.root);
        ew_absorbed_[C.root] = 1;
        ew_post_[C.root] = 1;
        ew_group_[C.root] = -1;
        C.root = -1;
      }
    }
    R.post.assign(post.begin(), post.end());
  }

  // Epilogue groups: a group over the row reduction's input shape that reads
  // the reduction's per-row results (or its post ops'), and otherwise only
  // tensors stored before the reduction in plain index modes, is evaluated by
  // the row's warp right after the row values: one launch and one pass over
  // the rows less (LayerNorm's normalisation, its gradient's dx).
  for (size_t ri = 0; ri < ew_groups_.size(); ++ri) {
    EwGroup& R = ew_groups_[ri];
    if (R.red < 0 || R.epi_root >= 0) continue;
    int64_t rows = 0, len = 0;
    if (red_shape(P, R.red, &rows, &len) != RED_ROW || len > kWarpRowMax) continue;
    const int t = P.out[R.red];
    if (P.T[t].numel != rows) continue;
    const auto& vshape = P.T[P.op(R.red)["a"].i32()].shape;
    std::set<int> rowvals;
    for (const auto& kv : row_values(R)) rowvals.insert(kv.first);
    bool done_r = false;
    for (int rv : rowvals) {
      for (int c : P.consumers[rv]) {
        auto it = owners.find(c);
        if (it == owners.end()) continue;
        for (int ci : it->second) {
          EwGroup& C = ew_groups_[ci];
          if (ci == (int)ri || C.red >= 0 || C.root < 0 || ew_group_[C.root] != ci) continue;
          if (P.T[P.out[C.root]].shape != vshape || side(C.root) != side(R.red)) continue;
          if ((int)C.members.size() > kMaxGroupOps) continue;
          const std::set<int> cm(C.members.begin(), C.members.end());
          bool ok = true;
          for (int m : C.members)
            for (int x : ew_operands(P, m)) {
              if (rowvals.count(x)) {
                if (!reads_as_row(x, vshape, len)) ok = false;
                continue;
              }
              if (cm.count(P.producer[x])) continue;
              const TView& vx = views_[x];
              if (vx.onehot || ew_internal(x) || P.producer[x] >= R.red) { ok = false; continue; }
              bool dummy = true;
              const int mode = ew_input(x, vshape, dummy, false).mode;
              if (mode != IN_FULL && mode != IN_SCALAR && mode != IN_PERIOD && mode != IN_ROWDIV) ok = false;
            }
          if (!ok) continue;
          R.epi = C.members;
          R.epi_root = C.root;
          ew_absorbed_[C.root] = 1;
          ew_post_[C.root] = 1;
          ew_group_[C.root] = -1;
          C.root = -1;
          done_r = true;
          break;
        }
        if (done_r) break;
      }
      if (done_r) break;
    }
  }

  // A dropout that is the only member of its group and reads a causal
  // softmax's result is written by the softmax kernel as a second output
  // (attention's dropout on the probabilities): one read of the [.., T, T]
  // tensor less.
  softmax_drop_.clear();
  extra_writes_.clear();
  for (int sm = 0; sm < nO; ++sm) {
    if (op_done_[sm] || action_[sm] != 0 || P.kind[sm] != "softmax_causal_last") continue;
    const int pt = P.out[sm];
    if (P.T[pt].shape.back() > 1024 || views_[pt].root != pt || !views_[pt].contiguous) continue;
    for (int d : P.consumers[pt]) {
      const int gi = ew_group_of(d);
      if (P.kind[d] != "dropout" || gi < 0 || ew_groups_[gi].members != std::vector<int>{d}) continue;
      const int dt = P.out[d];
      if (P.T[dt].shape != P.T[pt].shape || views_[dt].root != dt || !views_[dt].contiguous) continue;
      if (side(d) != side(sm)) continue;
      softmax_drop_[sm] = d;
      extra_writes_[sm].push_back(dt);
      ew_group_[d] = -1;
      ew_absorbed_[d] = 1;
      ew_post_[d] = 1;
      ew_groups_[gi].root = -1;
      break;
    }
  }

  // A plain row mean / sum of a stored tensor whose result a fused row
  // reduction over the same rows reads later in the step (LayerNorm: the
  // mean, then the variance of x - mean, then the normalisation) is computed
  // by that reduction's kernel as a first pass over each row: one launch and
  // one read of the mean less. Every reader of the result must run in that
  // launch or after it, and its aliases must be views.
  for (size_t ri = 0; ri < ew_groups_.size(); ++ri) {
    EwGroup& R = ew_groups_[ri];
    if (R.red < 0 || R.root < 0 || R.pre >= 0) continue;
    int64_t rows = 0, len = 0;
    if (red_shape(P, R.red, &rows, &len) != RED_ROW || len > kWarpRowMax) continue;
    const auto& vshape = P.T[P.op(R.red)["a"].i32()].shape;
    std::set<int> readers(R.members.begin(), R.members.end());
    readers.insert(R.post.begin(), R.post.end());
    readers.insert(R.epi.begin(), R.epi.end());
    for (int m : R.members) {
      for (int x : ew_operands(P, m)) {
        int b = x;
        while (P.producer[b] >= 0 && (P.kind[P.producer[b]] == "reshape" || P.kind[P.producer[b]] == "stop_gradient")) {
          const int src = P.op(P.producer[b])["a"].i32();
          if (P.T[src].numel != P.T[b].numel) break;
          b = src;
        }
        const int r1 = P.producer[b];
        if (r1 < 0 || r1 >= R.red || op_done_[r1] || action_[r1] != 0 || ew_group_of(r1) >= 0) continue;
        if (P.kind[r1] != "mean_last" && P.kind[r1] != "sum_last") continue;
        int64_t rows1 = 0, len1 = 0;
        if (red_shape(P, r1, &rows1, &len1) != RED_ROW || rows1 != rows || len1 != len) continue;
        const int a1 = P.op(r1)["a"].i32();
        if (views_[a1].onehot || ew_internal(a1) || P.T[a1].shape != vshape) continue;
        bool dummy = true;
        if (ew_input(a1, vshape, dummy, false).mode != IN_FULL) continue;
        bool ok = views_[b].root == b;
        const std::set<int> row_readers = [&] {
          std::set<int> s(R.members.begin(), R.members.end());
          s.insert(R.epi.begin(), R.epi.end());
          return s;
        }();
        for (int y : view_aliases(P, b))
          for (int c : P.consumers[y]) {
            const bool alias = (P.kind[c] == "reshape" || P.kind[c] == "stop_gradient") &&
                               P.T[P.out[c]].numel == P.T[y].numel;
            if (alias ? !op_done_[c] : (!readers.count(c) && c <= R.red)) ok = false;
            // the kernel hands every reader the row's value from a register,
            // so each alias read over the row shape must index per row
            if (!alias && row_readers.count(c) && !reads_as_row(y, vshape, len)) ok = false;
          }
        if (!ok) continue;
        R.pre = r1;
        op_done_[r1] = 1;
        extra_writes_[R.red].push_back(b);
        break;
      }
      if (R.pre >= 0) break;
    }
  }

  // A plain column sum of a tensor that an elementwise group writes and other
  // ops also read (a bias gradient of a stored activation gradient) is
  // computed by that group's launch as it stores the tensor: the launch runs
  // at the group's position and becomes a column reduction that also writes
  // its per-element value. One launch and one read of the tensor less.
  wt_reds_.clear();
  for (int r = 0; r < nO; ++r) {
    if (op_done_[r] || action_[r] != 0 || P.kind[r] != "sum_to_shape" || ew_group_of(r) >= 0) continue;
    int64_t rows = 0, len = 0;
    if (red_shape(P, r, &rows, &len) != RED_COL) continue;
    const int a = P.op(r)["a"].i32(), q = P.producer[a];
    if (q < 0 || side(q) != side(r)) continue;
    const int gi = ew_group_of(q);
    if (gi < 0) continue;
    EwGroup& G = ew_groups_[gi];
    if (G.red >= 0 || G.root != q || G.wt >= 0 || (int)G.members.size() > kMaxGroupOps) continue;
    // large arithmetic-heavy groups (erf, exp, division) keep the elementwise
    // grid's full occupancy: as a column reduction (four blocks per SM) the
    // GELU gradient of a [16384, 1536] tensor measured 94 us against 62 + 30 us
    // for the two launches. Small tensors are launch-bound and merge.
    bool heavy = false;
    for (int m : G.members) heavy = heavy || expensive_kind(P.kind[m]);
    if (heavy && P.T[a].numel >= (int64_t(1) << 22)) continue;
    if (views_[a].root != a || !views_[a].contiguous || views_[a].onehot) continue;
    G.wt = q;
    G.red = r;
    G.root = r;
    op_done_[r] = 1;
    wt_reds_.insert(r);
    extra_writes_[q].push_back(P.out[r]);
  }
}

namespace {

// Per-lane CUDA expression of one elementwise op over operand expressions.
std::string ew_expr(const Program& P, int i, const std::vector<std::string>& a, bool int_cmp) {
  const std::string& k = P.kind[i];
  const auto& O = P.op(i);
  auto bin = [&](const char* f) { return std::string(f) + "(" + a[0] + ", " + a[1] + ")"; };
  if (k == "add") return bin("__fadd_rn");
  if (k == "sub") return bin("__fsub_rn");
  if (k == "mul") return bin("__fmul_rn");
  if (k == "div") return bin("__fdiv_rn");
  if (k == "min") return bin("fminf");
  if (k == "max") return bin("fmaxf");
  if (k == "less" || k == "greater") {
    const char* op = k == "less" ? " < " : " > ";
    std::string x = int_cmp ? "__float_as_int(" + a[0] + ")" : a[0];
    std::string y = int_cmp ? "__float_as_int(" + a[1] + ")" : a[1];
    return "((" + x + op + y + ") ? tg_bits(1u) : tg_bits(0u))";
  }
  if (k == "sqrt") return "__fsqrt_rn(" + a[0] + ")";
  if (k == "rsqrt") return "__fdiv_rn(1.0f, __fsqrt_rn(" + a[0] + "))";
  if (k == "log") return "logf(" + a[0] + ")";
  if (k == "exp") return "expf(" + a[0] + ")";
  if (k == "relu") return "fmaxf(" + a[0] + ", 0.f)";
  if (k == "neg") return "(-" + a[0] + ")";
  if (k == "abs") return "fabsf(" + a[0] + ")";
  if (k == "tanh") return "tanhf(" + a[0] + ")";
  if (k == "sigmoid") return "(0.5f + 0.5f * tanhf(0.5f * " + a[0] + "))";
  if (k == "erf") return "tg_erf(" + a[0] + ")";
  if (k == "sin") return "sinf(" + a[0] + ")";
  if (k == "cos") return "cosf(" + a[0] + ")";
  if (k == "mul_scalar") return "__fmul_rn(" + a[0] + ", " + lit((float)O["scalar"].num()) + ")";
  if (k == "add_scalar") return "__fadd_rn(" + a[0] + ", " + lit((float)O["scalar"].num()) + ")";
  if (k == "broadcast_to") return a[0];
  if (k == "where_causal") {
    std::string T = std::to_string(P.T[P.out[i]].shape.back()) + "ll";
    return "(((e % " + T + ") > ((e / " + T + ") % " + T + ")) ? " + lit((float)O["fillValue"].num()) + " : " + a[0] + ")";
  }
  if (k == "dropout") {
    // src/codegen.ts:241-268: keep when u32 hash / 2^32 >= p, scale by 1/(1-p)
    double p = O["p"].num();
    uint32_t salt = (uint32_t)(((uint64_t)O["salt"].i64() * 0x9E3779B1ull) & 0xFFFFFFFFull);
    char buf[64];
    snprintf(buf, sizeof buf, "0x%08xu", salt);
    return "__fmul_rn(" + a[0] + ", (__uint2float_rn(tg_pcg(seed ^ " + buf + " ^ (u32)(drop_off + e))) * " +
           "2.3283064365386963e-10f >= " + lit(f32_lit8(p)) + ") ? " + lit(f32_lit8(1.0 / (1.0 - p))) + " : 0.f)";
  }
  if (k == "where") return "((__float_as_int(" + a[0] + ") != 0) ? " + a[1] + " : " + a[2] + ")";
  if (k == "relu_grad") return "((" + a[0] + " > 0.f) ? " + a[1] + " : 0.f)";
  if (k == "adam_update_m" || k == "adam_update_v") {
    double beta = O[k == "adam_update_m" ? "beta1" : "beta2"].num();
    std::string b = lit((float)beta), c = lit((float)(1.0 - beta));
    if (k == "adam_update_m") return "__fadd_rn(__fmul_rn(" + b + ", " + a[0] + "), __fmul_rn(" + c + ", " + a[1] + "))";
    return "__fadd_rn(__fmul_rn(" + b + ", " + a[0] + "), __fmul_rn(__fmul_rn(" + c + ", " + a[1] + "), " + a[1] + "))";
  }
  if (k == "adam_update_p") {
    // operands: p, mNew, lrt, [shrink], vNew
    bool has_sh = a.size() == 5;
    std::string sh = has_sh ? a[3] : lit((float)O["decayShrink"].num());
    std::string v = a[has_sh ? 4 : 3];
    return "__fsub_rn(__fmul_rn(" + sh + ", " + a[0] + "), __fdiv_rn(__fmul_rn(" + a[2] + ", " + a[1] +
           "), __fadd_rn(__fsqrt_rn(" + v + "), " + lit((float)O["eps"].num()) + ")))";
  }
  throw TgError("Error", "internal: no fused form for " + k);
}

}  // namespace

void Graph::emit_ew_group(int gi, const int* seed_ptr, float* scratch, size_t scratch_floats,
                          const std::function<void(const std::string&, std::function<void(cudaStream_t)>)>& add) {
  const EwGroup& G = ew_groups_[gi];
  const std::set<int> member_set(G.members.begin(), G.members.end());
  // The elementwise value the group produces: the root's output, or the
  // reduction's input. Every member is evaluated at that value's shape.
  const int vt = G.red >= 0 ? P.op(G.red)["a"].i32() : P.out[G.root];
  const auto& os = P.T[vt].shape;
  const int64_t n = P.T[vt].numel;
  if (n <= 0) return;
  int64_t rows = 0, len = 0;
  const RedShape rs = G.red >= 0 ? red_shape(P, G.red, &rows, &len) : RED_NONE;
  if (G.red >= 0 && rs == RED_NONE) throw TgError("Error", "internal: fused reduction of an unsupported shape");
  // float4 form: plain elementwise groups, and column sums over rows whose
  // length is a multiple of 4 (four adjacent columns per thread)
  bool vec = rs == RED_NONE || (rs == RED_COL && len % 4 == 0);
  std::vector<EwInput> ins;
  std::set<int> reads;  // distinct tensors the launch reads, for its byte count
  std::map<int, int> slot_of;
  bool has_drop = false;
  std::ostringstream ops;
  std::string label;
  // the first-pass row value (and its views), a register in the row loop
  const std::set<int> pre_vals = G.pre >= 0 ? view_aliases(P, P.out[G.pre]) : std::set<int>{};
  int pre_slot = -1;
  if (G.pre >= 0) {
    pre_slot = (int)ins.size();
    ins.push_back(ew_input(P.op(G.pre)["a"].i32(), os, vec));
    reads.insert(P.op(G.pre)["a"].i32());
    slot_of.emplace(P.op(G.pre)["a"].i32(), pre_slot);
  }
  for (int m : G.members) {
    std::vector<std::string> a;
    for (int t : ew_operands(P, m)) {
      if (member_set.count(P.producer[t]) || pre_vals.count(t)) { a.push_back("v" + std::to_string(t)); continue; }
      auto it = slot_of.find(t);
      if (it == slot_of.end()) {
        it = slot_of.emplace(t, (int)ins.size()).first;
        ins.push_back(ew_input(t, os, vec));
        reads.insert(t);
      }
      a.push_back("x" + std::to_string(it->second));
    }
    bool int_cmp = (P.kind[m] == "less" || P.kind[m] == "greater") && P.T[ew_operands(P, m)[0]].dtype != F32;
    if (P.kind[m] == "dropout") has_drop = true;
    if ((P.kind[m] == "add" || P.kind[m] == "sub" || P.kind[m] == "mul" || P.kind[m] == "div" ||
         P.kind[m] == "min" || P.kind[m] == "max") && P.T[P.out[m]].dtype != F32)
      throw TgError("Error", P.kind[m] + ": only f32 arithmetic is supported");
    ops << "      const float v" << P.out[m] << " = " << ew_expr(P, m, a, int_cmp) << ";\n";
    if (!label.empty()) label += "+";
    label += P.kind[m];
  }
  const std::string value = "v" + std::to_string(vt);
  void* out = ptr(P.out[G.root]);
  if (rs == RED_NONE) vec = vec && n % 4 == 0 && ((uintptr_t)out & 15) == 0;
  const int64_t col_chunks = rs == RED_COL ? colsum_chunks(rows, len) : 1;
  const int R = (int)os.size();

  // Register-cached rows (warp-per-row reductions over rows of 32·KJ
  // elements): each lane loads its KJ elements of every full-size input once
  // per row into registers, all loads of a row in flight together, and every
  // pass over the row (first-pass mean, the reduction, the epilogue) reads
  // them from there; inputs that repeat along rows (LayerNorm's gain and
  // bias) are loaded once per warp, per-row scalars once per row. The
  // arithmetic and its order are the uncached kernel's, so results are
  // bit-identical.
  const bool rowc = rs == RED_ROW && len <= kWarpRowMax && len % 32 == 0;
  const int64_t KJ = rowc ? len / 32 : 0;
  int64_t cache_budget = rowc ? 72 : 0;  // cached floats per lane
  std::vector<int> cmode;                // per slot: 0 load, 1 row array, 2 column array, 3 row scalar
  auto cache_slot = [&](int si) {
    if ((int)cmode.size() <= si) cmode.resize(si + 1, 0);
    if (!rowc) return;
    const EwInput& in = ins[si];
    if (in.mode == IN_ROWDIV && in.period == len) cmode[si] = 3;
    else if ((in.mode == IN_FULL || (in.mode == IN_PERIOD && in.period == len)) && cache_budget >= KJ) {
      cmode[si] = in.mode == IN_FULL ? 1 : 2;
      cache_budget -= KJ;
    }
  };
  auto cached_ref = [&](int si) -> std::string {
    return cmode[si] == 3 ? "s" + std::to_string(si) : "c" + std::to_string(si) + "[jj]";
  };
  if (pre_slot >= 0) cache_slot(pre_slot);

  // Per-element values of each input: for the vector form, loads before the
  // 4-lane loop plus per-lane picks; otherwise one load per element index e.
  std::ostringstream pre, lane;
  for (size_t si = 0; si < ins.size(); ++si) {
    const EwInput& in = ins[si];
    std::string p = "p" + std::to_string(si), x = "x" + std::to_string(si);
    std::string per = std::to_string(in.period) + "ll";
    if ((int)si != pre_slot) cache_slot((int)si);
    if (cmode[si]) {
      lane << "      const float " << x << " = " << cached_ref((int)si) << ";\n";
      continue;
    }
    switch (in.mode) {
      case IN_FULL:
        if (vec) { pre << "    const float4 q" << si << " = __ldg(reinterpret_cast<const float4*>(" << p << " + i));\n";
                   lane << "      const float " << x << " = f4(q" << si << ", l);\n"; }
        else lane << "      const float " << x << " = __ldg(" << p << " + e);\n";
        break;
      case IN_SCALAR:
        lane << "      const float " << x << " = __ldg(" << p << ");\n";
        break;
      case IN_PERIOD:
        if (vec) { pre << "    const float4 q" << si << " = __ldg(reinterpret_cast<const float4*>(" << p << " + i % " << per << "));\n";
                   lane << "      const float " << x << " = f4(q" << si << ", l);\n"; }
        else lane << "      const float " << x << " = __ldg(" << p << " + e % " << per << ");\n";
        break;
      case IN_ROWDIV:
        if (vec) { pre << "    const float s" << si << " = __ldg(" << p << " + i / " << per << ");\n";
                   lane << "      const float " << x << " = s" << si << ";\n"; }
        else lane << "      const float " << x << " = __ldg(" << p << " + e / " << per << ");\n";
        break;
      case IN_ONEHOT:
        lane << "      const float " << x << " = ((i64)__ldg(reinterpret_cast<const int*>(" << p << ") + e / " << per
             << ") == e % " << per << ") ? 1.f : 0.f;\n";
        break;
      default: {  // IN_STRIDED: row-major coordinates of e, dotted with the operand's strides
        lane << "      i64 o" << si << " = 0;\n      { i64 rem = e;\n";
        for (int d = R - 1; d >= 0; --d) {
          if (os[d] == 1) continue;
          if (in.strides[d] != 0)
            lane << "        o" << si << " += (rem % " << os[d] << "ll) * " << in.strides[d] << "ll;\n";
          if (d > 0) lane << "        rem /= " << os[d] << "ll;\n";
        }
        lane << "      }\n      const float " << x << " = __ldg(" << p << " + o" << si << ");\n";
      }
    }
  }

  // Post ops (row reductions): evaluated by lane 0 on the row's result; their
  // other inputs are per-row tensors (read at the row) or scalars.
  std::ostringstream post, post_w, epi;
  const bool has_post = rs == RED_ROW && !G.post_roots.empty();
  const bool has_epi = rs == RED_ROW && G.epi_root >= 0;
  if (has_post) {
    const int t = P.out[G.red];
    const std::set<int> pm(G.post.begin(), G.post.end());
    std::map<int, int> pslot;
    for (int m : G.post) {
      std::vector<std::string> a;
      for (int x : ew_operands(P, m)) {
        if (x == t || pm.count(P.producer[x]) || pre_vals.count(x)) { a.push_back("v" + std::to_string(x)); continue; }
        auto it = pslot.find(x);
        if (it == pslot.end()) {
          it = pslot.emplace(x, (int)ins.size()).first;
          EwInput in{};
          in.ptr = ptr(x);
          in.mode = P.T[x].numel == 1 ? IN_SCALAR : IN_FULL;
          ins.push_back(in);
          reads.insert(x);
          cmode.resize(ins.size(), 0);
          post << "      const float y" << it->second << " = __ldg(p" << it->second
               << (P.T[x].numel == 1 ? ")" : " + r)") << ";\n";
        }
        a.push_back("y" + std::to_string(it->second));
      }
      const bool int_cmp = (P.kind[m] == "less" || P.kind[m] == "greater") && P.T[ew_operands(P, m)[0]].dtype != F32;
      post << "      const float v" << P.out[m] << " = " << ew_expr(P, m, a, int_cmp) << ";\n";
    }
    for (size_t pr = 0; pr < G.post_roots.size(); ++pr)
      post_w << "      out" << 2 + pr << "[r] = v" << P.out[G.post_roots[pr]] << ";\n";
    label += "+post:";
    for (int m : G.post) label += P.kind[m] + (m == G.post.back() ? "" : "+");
  }
  if (has_epi) {
    const std::map<int, int> rva = row_values(G);
    std::set<int> rowvals;
    for (const auto& kv : rva)
      if (rowvals.insert(kv.first).second && kv.first != kv.second)
        epi << "        const float v" << kv.first << " = v" << kv.second << ";\n";
    const std::set<int> em(G.epi.begin(), G.epi.end());
    std::map<int, int> eslot;
    for (int m : G.epi) {
      std::vector<std::string> a;
      for (int x : ew_operands(P, m)) {
        if (rowvals.count(x) || em.count(P.producer[x]) || pre_vals.count(x)) { a.push_back("v" + std::to_string(x)); continue; }
        auto it = eslot.find(x);
        if (it == eslot.end()) {
          bool dummy = true;
          EwInput in = ew_input(x, os, dummy);
          auto shared = slot_of.find(x);  // an input the row pass reads already
          if (shared != slot_of.end()) {
            it = eslot.emplace(x, shared->second).first;
          } else {
            it = eslot.emplace(x, (int)ins.size()).first;
            ins.push_back(in);
            reads.insert(x);
            cache_slot(it->second);
          }
          const int es = it->second;
          const std::string pp = "p" + std::to_string(es), per = std::to_string(in.period) + "ll";
          std::string ld;
          if (cmode[es]) ld = cached_ref(es);
          else if (in.mode == IN_FULL) ld = "__ldg(" + pp + " + e)";
          else if (in.mode == IN_SCALAR) ld = "__ldg(" + pp + ")";
          else if (in.mode == IN_PERIOD) ld = "__ldg(" + pp + " + e % " + per + ")";
          else ld = "__ldg(" + pp + " + e / " + per + ")";
          epi << "        const float z" << it->second << " = " << ld << ";\n";
        }
        a.push_back("z" + std::to_string(it->second));
      }
      if (P.kind[m] == "dropout") has_drop = true;
      const bool int_cmp = (P.kind[m] == "less" || P.kind[m] == "greater") && P.T[ew_operands(P, m)[0]].dtype != F32;
      epi << "        const float v" << P.out[m] << " = " << ew_expr(P, m, a, int_cmp) << ";\n";
    }
    epi << "        oute[e] = v" << P.out[G.epi_root] << ";\n";
    label += "+epi:";
    for (int m : G.epi) label += P.kind[m] + (m == G.epi.back() ? "" : "+");
  }

  std::ostringstream k;
  k << "(";
  for (size_t si = 0; si < ins.size(); ++si) k << "const float* __restrict__ p" << si << ", ";
  k << "float* __restrict__ out, ";
  if (has_post)
    for (size_t pr = 0; pr < G.post_roots.size(); ++pr) k << "float* __restrict__ out" << 2 + pr << ", ";
  if (has_epi) k << "float* __restrict__ oute, ";
  if (G.pre >= 0) k << "float* __restrict__ outp, ";
  if (G.wt >= 0) k << "float* __restrict__ outw, ";
  k << "const int* __restrict__ seedp, i64 drop_off) {\n";
  k << "  const u32 seed = " << (has_drop ? "seedp ? (u32)(*seedp) : 0u" : "0u") << ";\n";
  k << "  (void)seed; (void)drop_off;\n";
  int64_t nchunk = 1;
  const std::string L = std::to_string(len) + "ll";
  if (rs == RED_ROW && len > kWarpRowMax) {
    // one block per row: thread t sums j = t, t + 256, ..., then warp trees and
    // the 8 warp sums in order (a fixed order, so deterministic)
    const bool mean = P.kind[G.red] == "mean_last";
    k << "  __shared__ float wsum[8];\n  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;\n";
    k << "  for (i64 r = blockIdx.x; r < " << rows << "ll; r += gridDim.x) {\n";
    k << "    float acc = 0.f;\n#pragma unroll 4\n    for (i64 j = threadIdx.x; j < " << L << "; j += 256) {\n      const i64 e = r * "
      << L << " + j;\n";
    k << lane.str() << ops.str() << "      acc += " << value << ";\n    }\n";
    k << "    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);\n";
    k << "    if (lane == 0) wsum[wid] = acc;\n    __syncthreads();\n";
    k << "    if (threadIdx.x == 0) {\n      float t = 0.f;\n      for (int w = 0; w < 8; ++w) t += wsum[w];\n";
    k << "      out[r] = " << (mean ? "__fdiv_rn(t, " + lit((float)len) + ")" : "t") << ";\n    }\n    __syncthreads();\n  }\n}\n";
  } else if (rs == RED_ROW) {
    // one warp per row; lanes sum j = lane, lane + 32, ... then a shuffle tree
    // (the unfused row kernel's order)
    const bool mean = P.kind[G.red] == "mean_last";
    k << "  const int lane = threadIdx.x & 31;\n  const i64 nw = ((i64)gridDim.x * 256) >> 5;\n";
    // the loop over a row's elements: fully unrolled over the lane's KJ
    // cached elements, or the plain strided loop
    auto row_loop = [&](const char* ind) {
      std::string s = ind;
      if (rowc)
        return s + "#pragma unroll\n" + s + "for (int jj = 0; jj < " + std::to_string(KJ) + "; ++jj) {\n" + s +
               "  const i64 j = lane + 32 * jj;\n";
      return s + "for (i64 j = lane; j < " + L + "; j += 32) {\n";
    };
    for (size_t si = 0; si < cmode.size(); ++si)
      if (cmode[si] == 2)
        k << "  float c" << si << "[" << KJ << "];\n#pragma unroll\n  for (int jj = 0; jj < " << KJ << "; ++jj) c" << si
          << "[jj] = __ldg(p" << si << " + lane + 32 * jj);\n";
    k << "  for (i64 r = (((i64)blockIdx.x * 256 + threadIdx.x) >> 5); r < " << rows << "ll; r += nw) {\n";
    for (size_t si = 0; si < cmode.size(); ++si) {
      if (cmode[si] == 1)
        k << "    float c" << si << "[" << KJ << "];\n#pragma unroll\n    for (int jj = 0; jj < " << KJ << "; ++jj) c" << si
          << "[jj] = __ldg(p" << si << " + r * " << L << " + lane + 32 * jj);\n";
      if (cmode[si] == 3) k << "    const float s" << si << " = __ldg(p" << si << " + r);\n";
    }
    if (G.pre >= 0 && rowc) {
      const int b = P.out[G.pre];
      k << "    float accp = 0.f;\n" << row_loop("    ") << "      accp += "
        << (cmode[pre_slot] ? cached_ref(pre_slot) : "__ldg(p" + std::to_string(pre_slot) + " + r * " + L + " + j)")
        << ";\n    }\n";
      k << "    for (int o = 16; o > 0; o >>= 1) accp += __shfl_xor_sync(0xffffffffu, accp, o);\n";
      k << "    const float v" << b << " = "
        << (P.kind[G.pre] == "mean_last" ? "__fdiv_rn(accp, " + lit((float)len) + ")" : "accp") << ";\n";
      for (int y : pre_vals)
        if (y != b) k << "    const float v" << y << " = v" << b << ";\n";
      k << "    if (lane == 0) outp[r] = v" << b << ";\n";
    } else if (G.pre >= 0) {
      // first pass: the absorbed row reduction, in the same lane order and
      // tree as the row kernels; lane 0 stores it, every lane keeps it
      const int b = P.out[G.pre];
      k << "    float accp = 0.f;\n#pragma unroll 4\n    for (i64 j = lane; j < " << L << "; j += 32) accp += __ldg(p"
        << pre_slot << " + r * " << L << " + j);\n";
      k << "    for (int o = 16; o > 0; o >>= 1) accp += __shfl_xor_sync(0xffffffffu, accp, o);\n";
      k << "    const float v" << b << " = "
        << (P.kind[G.pre] == "mean_last" ? "__fdiv_rn(accp, " + lit((float)len) + ")" : "accp") << ";\n";
      for (int y : pre_vals)
        if (y != b) k << "    const float v" << y << " = v" << b << ";\n";
      k << "    if (lane == 0) outp[r] = v" << b << ";\n";
    }
    if (rowc) k << "    float acc = 0.f;\n" << row_loop("    ") << "      const i64 e = r * " << L << " + j;\n";
    else
      k << "    float acc = 0.f;\n#pragma unroll 4\n    for (i64 j = lane; j < " << L << "; j += 32) {\n      const i64 e = r * " << L
        << " + j;\n";
    k << lane.str() << ops.str() << "      acc += " << value << ";\n    }\n";
    k << "    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);\n";
    const std::string red = mean ? "__fdiv_rn(acc, " + lit((float)len) + ")" : "acc";
    if (has_post || has_epi) {
      // every lane holds the row sum (xor tree): the row values are computed
      // on all lanes, lane 0 stores them, the epilogue runs over the row
      k << "    {\n      const float v" << P.out[G.red] << " = " << red << ";\n" << post.str();
      k << "      if (lane == 0) {\n        out[r] = v" << P.out[G.red] << ";\n" << post_w.str() << "      }\n";
      if (has_epi)
        k << row_loop("      ") << "        const i64 e = r * " << L << " + j;\n" << epi.str() << "      }\n";
      k << "    }\n  }\n}\n";
    } else {
      k << "    if (lane == 0) out[r] = " << red << ";\n  }\n}\n";
    }
  } else if (rs == RED_COL) {
    // first pass of the deterministic column sum: rows of chunk blockIdx.y in
    // ascending order (the unfused kernel's order); the fold is shared
    nchunk = col_chunks;
    if (nchunk > 1 && (!scratch || scratch_floats < (size_t)(nchunk * len)))
      throw TgError("Error", "internal: scratch too small for a fused column sum");
    const int64_t rp = (rows + nchunk - 1) / nchunk;
    // 32 column threads (4 adjacent columns each in the float4 form) x 8 row
    // groups, combined in group order: the unfused column sum's order
    const int W = vec ? 4 : 1;
    k << "  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;\n";
    k << "  __shared__ float red[8][" << 32 * W << "];\n";
    k << "  const i64 col = ((i64)blockIdx.x * 32 + tx) * " << W << ";\n";
    k << "  const i64 r0 = (i64)blockIdx.y * " << rp << "ll;\n";
    k << "  const i64 r1 = r0 + " << rp << "ll < " << rows << "ll ? r0 + " << rp << "ll : " << rows << "ll;\n";
    k << "  float acc[" << W << "];\n  for (int l = 0; l < " << W << "; ++l) acc[l] = 0.f;\n";
    k << "  if (col < " << L << ") {\n#pragma unroll 4\n    for (i64 r = r0 + ty; r < r1; r += 8) {\n";
    if (vec) {
      k << "    const i64 i = r * " << L << " + col;\n" << pre.str();
      if (G.wt >= 0) k << "    float w4[4];\n";
      k << "#pragma unroll\n    for (int l = 0; l < 4; ++l) {\n      const i64 e = i + l;\n";
      k << lane.str() << ops.str() << "      acc[l] += " << value << ";\n";
      if (G.wt >= 0) k << "      w4[l] = " << value << ";\n";
      k << "    }\n";
      if (G.wt >= 0) k << "    *reinterpret_cast<float4*>(outw + i) = make_float4(w4[0], w4[1], w4[2], w4[3]);\n";
    } else {
      k << "      const i64 e = r * " << L << " + col;\n";
      k << lane.str() << ops.str() << "      acc[0] += " << value << ";\n";
      if (G.wt >= 0) k << "      outw[e] = " << value << ";\n";
    }
    k << "    }\n  }\n";
    k << "  for (int l = 0; l < " << W << "; ++l) red[ty][tx * " << W << " + l] = acc[l];\n  __syncthreads();\n";
    k << "  if (ty == 0 && col < " << L << ") {\n    for (int l = 0; l < " << W << "; ++l) {\n";
    k << "      float t = 0.f;\n#pragma unroll\n      for (int g = 0; g < 8; ++g) t += red[g][tx * " << W << " + l];\n";
    k << "      out[(i64)blockIdx.y * " << L << " + col + l] = t;\n    }\n  }\n}\n";
  } else if (vec) {
    k << "  for (i64 t = (i64)blockIdx.x * 256 + threadIdx.x; t < " << n / 4 << "ll; t += (i64)gridDim.x * 256) {\n";
    k << "    const i64 i = t * 4;\n" << pre.str();
    k << "    float r[4];\n#pragma unroll\n    for (int l = 0; l < 4; ++l) {\n      const i64 e = i + l;\n";
    k << lane.str() << ops.str() << "      r[l] = " << value << ";\n    }\n";
    k << "    *reinterpret_cast<float4*>(out + i) = make_float4(r[0], r[1], r[2], r[3]);\n  }\n}\n";
  } else {
    k << "  for (i64 e = (i64)blockIdx.x * 256 + threadIdx.x; e < " << n << "ll; e += (i64)gridDim.x * 256) {\n";
    k << pre.str() << lane.str() << ops.str() << "      out[e] = " << value << ";\n  }\n}\n";
  }
  std::string body = k.str();
  char name[40];
  snprintf(name, sizeof name, "tgew_%016zx", std::hash<std::string>{}(body));
  std::string src = std::string("extern \"C\" __global__ void __launch_bounds__(256) ") + name + body;
  std::shared_ptr<JitFn> fn;
  if (ctx->dry) {
    jit_sources_.push_back(src);
    fn = std::make_shared<JitFn>();
    fn->name = name;
  } else {
    fn = jit_request(name, src);
  }

  struct Args {
    std::vector<const void*> in;
    void* out;
    std::vector<void*> outs;  // post roots' outputs
    const int* seed;
    long long drop_off;
  };
  auto A = std::make_shared<Args>();
  for (auto& in : ins) A->in.push_back(in.ptr);
  if (has_post)
    for (int pr : G.post_roots) A->outs.push_back(ptr(P.out[pr]));
  if (has_epi) A->outs.push_back(ptr(P.out[G.epi_root]));
  if (G.pre >= 0) A->outs.push_back(ptr(P.out[G.pre]));
  if (G.wt >= 0) A->outs.push_back(ptr(P.out[G.wt]));
  A->out = (rs == RED_COL && nchunk > 1) ? static_cast<void*>(scratch) : out;
  A->seed = seed_ptr;
  A->drop_off = (long long)ctx->rank * n;
  const int64_t sms = device_sm_count();
  unsigned gx = 1, gy = 1;
  int tpb = 256;
  if (rs == RED_ROW && len > kWarpRowMax) {
    gx = (unsigned)std::max<int64_t>(1, std::min<int64_t>(rows, sms * 8));
  } else if (rs == RED_ROW) {
    const int64_t blocks = (rows + 7) / 8;
    gx = (unsigned)std::max<int64_t>(1, std::min(blocks, sms * 16));
  } else if (rs == RED_COL) {
    gx = (unsigned)colsum_col_blocks(len, vec);
    gy = (unsigned)nchunk;
  } else {
    const int64_t work = vec ? n / 4 : n;
    const int64_t blocks = (work + 255) / 256;
    gx = (unsigned)std::max<int64_t>(1, std::min(blocks, sms * 8));
  }
  if (G.red >= 0)
    label = "fused_red|" + (G.pre >= 0 ? P.kind[G.pre] + ">" : std::string()) + P.kind[G.red] +
            (G.wt >= 0 ? "+store" : "") + ":" + label.substr(0, 150);
  else if (G.members.size() > 1) label = "fused_ew|" + label.substr(0, 160);
  // algorithmic bytes: each distinct input once, every output once
  {
    double b = 0;
    for (int t : reads) b += tensor_bytes(t);
    b += tensor_bytes(P.out[G.root]);
    if (has_post) for (int pr : G.post_roots) b += tensor_bytes(P.out[pr]);
    if (has_epi) b += tensor_bytes(P.out[G.epi_root]);
    if (G.pre >= 0) b += tensor_bytes(P.out[G.pre]);
    if (G.wt >= 0) b += tensor_bytes(P.out[G.wt]);
    next_bytes_ = b;
  }
  float* fold_out = reinterpret_cast<float*>(out);
  const int64_t fold_n = (rs == RED_COL && nchunk > 1) ? nchunk : 0, fold_len = len;
  float* fold_part = scratch;
  add(label, [fn, A, gx, gy, tpb, fold_n, fold_len, fold_part, fold_out](cudaStream_t s) {
    std::vector<void*> args;
    for (auto& p : A->in) args.push_back(const_cast<const void**>(&p));
    args.push_back(&A->out);
    for (auto& o : A->outs) args.push_back(&o);
    args.push_back(const_cast<const int**>(&A->seed));
    args.push_back(&A->drop_off);
    jit_launch(*fn, gx, gy, tpb, args.data(), s);
    if (fold_n > 0) launch_colsum_fold(fold_part, fold_out, fold_n, fold_len, s);
  });
}

}  // namespace tg
