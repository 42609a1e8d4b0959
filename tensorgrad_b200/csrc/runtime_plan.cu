// Planner: wire program -> views, fused optimizer, storage arenas.
//
// Storage replaces the reference's planBuffers (src/buffers.ts:103-277):
// instead of one buffer per param/grad/state plus pooled intermediates, the
// planner lays params, their gradients and optimizer moments out as four
// flat arenas with one identical layout (so one fused kernel updates every
// parameter and one collective reduces every gradient), makes reshape-like
// ops zero-copy views, and packs intermediates into one arena by liveness
// (same best-fit idea and the same no-overlap invariant, checked below).
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <set>

#include "runtime.hpp"

namespace tg {

static int dtype_of(const std::string& s) {
  if (s == "f32") return F32;
  if (s == "i32") return I32;
  return BOOL;
}

void Program::parse(const char* json, size_t len) {
  root = tgjson::parse(json, len);
  const auto& g = root["graph"];
  const auto& ts = g["tensors"];
  T.resize(ts.size());
  for (size_t i = 0; i < ts.size(); ++i) {
    for (auto& d : ts[i]["shape"].a) T[i].shape.push_back(d.i64());
    T[i].dtype = dtype_of(ts[i]["dtype"].str());
    T[i].numel = 1;
    for (auto d : T[i].shape) T[i].numel *= d;
  }
  const auto& os = g["ops"];
  producer.assign(T.size(), -1);
  consumers.assign(T.size(), {});
  for (size_t i = 0; i < os.size(); ++i) {
    const auto& o = os[i];
    ops.push_back(&o);
    kind.push_back(o["kind"].str());
    int ot = o["out"].i32();
    out.push_back(ot);
    producer[ot] = (int)i;
    std::vector<int> in;
    const std::string& k = kind.back();
    auto add = [&](const char* f) { in.push_back(o[f].i32()); };
    static const std::set<std::string> leaf = {"param_input", "tensor_input", "state_input", "arange",
                                               "const_scalar", "const_fill"};
    static const std::set<std::string> ab = {"add", "sub", "mul", "div", "min", "max", "less", "greater",
                                             "matmul", "matmul_batched"};
    if (leaf.count(k)) {
    } else if (k == "randn") add("seed");
    else if (ab.count(k)) { add("a"); add("b"); }
    else if (k == "dropout" || k == "categorical_last") { add("a"); add("seed"); }
    else if (k == "one_hot") add("indices");
    else if (k == "where") { add("cond"); add("a"); add("b"); }
    else if (k == "concat") { for (auto& x : o["inputs"].a) in.push_back(x.i32()); }
    else if (k == "relu_grad") { add("x"); add("dy"); }
    else if (k == "adam_update_m") { add("m"); add("g"); }
    else if (k == "adam_update_v") { add("v"); add("g"); }
    else if (k == "adam_update_p") {
      add("p"); add("mNew"); add("vNew"); add("lrt");
      if (!o["decayShrinkTensor"].is_null()) add("decayShrinkTensor");
    }
    else if (k == "conv2d") { add("input"); add("weight"); }
    else if (k == "conv2d_input_grad") { add("weight"); add("dy"); }
    else if (k == "conv2d_weight_grad") { add("input"); add("dy"); }
    else if (k == "max_pool_2d") add("input");
    else if (k == "max_pool_2d_grad") { add("input"); add("dy"); }
    else add("a");
    for (int t : in) {
      auto& c = consumers[t];
      if (c.empty() || c.back() != (int)i) c.push_back((int)i);
    }
    op_inputs.push_back(std::move(in));
    if (k == "param_input") params.emplace_back(o["name"].str(), ot);
    if (k == "tensor_input") inputs[o["name"].str()] = ot;
  }
  for (auto& x : g["outputs"].a) outputs.push_back(x.i32());
  for (auto& kv : g["captures"].o) captures.emplace_back(kv.first, kv.second.i32());
  if (auto* st = root.find("states"))
    for (auto& kv : st->o) states.push_back({kv.first, kv.second["tensor"].i32(), kv.second["initValue"].num()});
  if (auto* pg = root.find("paramGrads"))
    for (auto& kv : pg->o) grads.emplace_back(kv.first, kv.second.i32());
  if (auto* wb = root.find("writebacks"))
    for (auto& w : wb->a) writebacks.push_back({w["source"].i32(), w["destName"].str(), w["destKind"].str() == "param"});
  if (auto* l = root.find("loss")) if (!l->is_null()) loss = l->i32();
  if (loss < 0 && !outputs.empty()) loss = outputs[0];
  opt_start = (int)ops.size();
  if (auto* s = root.find("optStart")) if (!s->is_null()) opt_start = s->i32();
  if (auto* o = root.find("optimizer")) if (!o->is_null()) optimizer = o;
  if (auto* u = root.find("usesPrng")) uses_prng = u->kind == tgjson::Value::Bool ? u->b : false;
}

static std::vector<int64_t> contig_strides(const std::vector<int64_t>& shape) {
  std::vector<int64_t> s(shape.size(), 1);
  for (int i = (int)shape.size() - 2; i >= 0; --i) s[i] = s[i + 1] * shape[i + 1];
  return s;
}

// ---------------------------------------------------------------- views ----
void Graph::plan_views() {
  const int nT = (int)P.T.size(), nO = (int)P.ops.size();
  views_.assign(nT, TView{});
  for (int t = 0; t < nT; ++t) {
    views_[t].root = t;
    views_[t].strides = contig_strides(P.T[t].shape);
  }
  std::set<int> pinned;  // tensors that must own storage (observable results)
  for (int t : P.outputs) pinned.insert(t);
  for (auto& c : P.captures) pinned.insert(c.second);
  for (auto& w : P.writebacks) pinned.insert(w.src);

  auto is_gemm = [&](int op) { return P.kind[op] == "matmul" || P.kind[op] == "matmul_batched"; };

  // Embedding patterns: matmul(one_hot(idx), table) -> row gather;
  // matmul(permute(reshape(one_hot(idx))), dy) -> sorted segmented sum.
  auto onehot_of = [&](int t) -> int {  // tensor id of the one_hot output feeding t, or -1
    int p = P.producer[t];
    if (p >= 0 && P.kind[p] == "one_hot" && P.T[t].dtype == F32) return t;
    return -1;
  };
  std::vector<int> gather_op, embgrad_op;  // op indices
  for (int i = 0; i < nO; ++i) {
    if (P.kind[i] != "matmul") continue;
    int a = P.op(i)["a"].i32(), b = P.op(i)["b"].i32();
    if (onehot_of(a) >= 0 && P.T[b].shape.size() == 2 &&
        P.op(P.producer[a])["depth"].i64() == P.T[b].shape[0]) {
      action_[i] = 100;  // gather
      continue;
    }
    int pa = P.producer[a];
    if (pa >= 0 && P.kind[pa] == "permute") {
      const auto& perm = P.op(pa)["perm"].a;
      int r = P.op(pa)["a"].i32();
      int pr = P.producer[r];
      if (perm.size() == 2 && perm[0].i32() == 1 && pr >= 0 && P.kind[pr] == "reshape" &&
          onehot_of(P.op(pr)["a"].i32()) >= 0 && P.T[r].shape.size() == 2 &&
          P.consumers[a].size() == 1 && P.consumers[r].size() == 1 && !pinned.count(a) && !pinned.count(r)) {
        action_[i] = 101;  // embedding grad
        op_done_[pa] = 1;
        op_done_[pr] = 1;
      }
    }
  }
  // One-hot stays virtual when every consumer reads it through a pattern
  // above or as a full-shape elementwise input.
  static const std::set<std::string> ew_kinds = {
      "add", "sub", "mul", "div", "min", "max", "mul_scalar", "add_scalar", "sqrt", "rsqrt", "log", "exp",
      "relu", "neg", "abs", "tanh", "sigmoid", "erf", "sin", "cos", "less", "greater", "where", "relu_grad",
      "dropout", "where_causal", "broadcast_to"};
  for (int i = 0; i < nO; ++i) {
    if (P.kind[i] != "one_hot") continue;
    int t = P.out[i];
    bool ok = !pinned.count(t) && P.T[t].dtype == F32;
    for (int c : P.consumers[t]) {
      if (!ok) break;
      if (action_[c] == 100) continue;
      if (P.kind[c] == "reshape" && op_done_[c]) continue;
      if (ew_kinds.count(P.kind[c]) && P.T[P.out[c]].shape == P.T[t].shape) continue;
      ok = false;
    }
    if (ok) {
      views_[t].onehot = true;
      views_[t].onehot_idx = P.op(i)["indices"].i32();
      op_done_[i] = 1;
    }
  }

  // sum_last(mul(x, oneHot(idx))) over a log-softmax x (the cross-entropy
  // gather): the row has one nonzero term, every other is x * 0 = 0 for the
  // finite x a log-softmax gives, so the sum is x[r, idx[r]] (0 when idx is
  // out of range), read directly instead of multiplying and summing the row.
  for (int r = 0; r < nO; ++r) {
    if (op_done_[r] || action_[r] != 0 || P.kind[r] != "sum_last") continue;
    const int a = P.op(r)["a"].i32(), m = P.producer[a];
    if (m < 0 || P.kind[m] != "mul" || op_done_[m] || pinned.count(a) || P.consumers[a].size() != 1) continue;
    int x = P.op(m)["a"].i32(), oh = P.op(m)["b"].i32();
    if (!views_[oh].onehot) std::swap(x, oh);
    if (!views_[oh].onehot || views_[x].onehot || !views_[x].contiguous) continue;
    if (P.T[x].shape != P.T[oh].shape || P.producer[x] < 0 || P.kind[P.producer[x]] != "log_softmax_last") continue;
    action_[r] = 102;
    op_done_[m] = 1;
  }

  // sum_last(mul(broadcast_to(g), oneHot(idx))) with g one value per row (the
  // cross-entropy gradient's one-hot term): the row sum is g[r] when idx[r] is
  // in range, else 0, formed without reading the [rows, V] product, which is
  // then left to its other consumers.
  for (int r = 0; r < nO; ++r) {
    if (op_done_[r] || action_[r] != 0 || P.kind[r] != "sum_last") continue;
    const int a = P.op(r)["a"].i32(), m = P.producer[a];
    if (m < 0 || P.kind[m] != "mul" || op_done_[m] || pinned.count(a)) continue;
    int u = P.op(m)["a"].i32(), oh = P.op(m)["b"].i32();
    if (!views_[oh].onehot) std::swap(u, oh);
    if (!views_[oh].onehot || views_[u].onehot) continue;
    const int pu = P.producer[u];
    if (pu < 0 || P.kind[pu] != "broadcast_to" || P.T[u].shape != P.T[oh].shape) continue;
    const int g = P.op(pu)["a"].i32();
    if (P.T[g].numel != P.T[P.out[r]].numel || views_[g].onehot || !views_[g].contiguous) continue;
    action_[r] = 103;
    no_read_.insert({r, a});
    if (P.consumers[a].size() == 1) op_done_[m] = 1;  // nothing else reads the product
  }

  // A permute is a view when everything that reads it takes strided operands:
  // GEMMs, or permutes that are views themselves (decided back to front).
  std::vector<char> pview(nO, 0);
  for (int i = nO - 1; i >= 0; --i) {
    if (op_done_[i] || P.kind[i] != "permute" || pinned.count(P.out[i])) continue;
    bool ok = !P.consumers[P.out[i]].empty();
    for (int c : P.consumers[P.out[i]])
      if (!((is_gemm(c) && action_[c] < 100) || (P.kind[c] == "permute" && pview[c]))) ok = false;
    pview[i] = ok;
  }

  // Zero-copy views, in op order so chains resolve.
  for (int i = 0; i < nO; ++i) {
    if (op_done_[i]) continue;
    const std::string& k = P.kind[i];
    int o = P.out[i];
    if (pinned.count(o)) continue;
    if (k == "reshape" || k == "stop_gradient" ||
        ((k == "sum_to_shape" || k == "broadcast_to") &&
         P.T[o].shape == P.T[P.op(i)["a"].i32()].shape)) {
      int a = P.op(i)["a"].i32();
      const TView& va = views_[a];
      if (va.onehot || !va.contiguous) continue;
      views_[o].root = va.root;
      views_[o].off = va.off;
      views_[o].contiguous = true;
      op_done_[i] = 1;
    } else if (k == "slice_range") {
      int a = P.op(i)["a"].i32();
      const TView& va = views_[a];
      if (va.onehot || !va.contiguous) continue;
      int ax = P.op(i)["axis"].i32();
      bool lead = true;
      for (int d = 0; d < ax; ++d) if (P.T[a].shape[d] != 1) lead = false;
      if (!lead) continue;
      views_[o].root = va.root;
      views_[o].off = va.off + P.op(i)["start"].i64() * va.strides[ax];
      views_[o].contiguous = true;
      op_done_[i] = 1;
    } else if (k == "permute") {
      int a = P.op(i)["a"].i32();
      const TView& va = views_[a];
      if (va.onehot) continue;
      if (!pview[i]) continue;
      const auto& perm = P.op(i)["perm"].a;
      views_[o].root = va.root;
      views_[o].off = va.off;
      views_[o].strides.clear();
      for (auto& pv : perm) views_[o].strides.push_back(va.strides[pv.i32()]);
      views_[o].contiguous = false;
      op_done_[i] = 1;
    }
  }

  // Producer-side views: a permute whose input is written by a GEMM (or by
  // another permute) and read by nothing else is done by that writer, which
  // stores straight into the permuted layout through its output strides
  // (attention's mergeHeads, and the head-split gradients). Back to front,
  // so a chain of permutes collapses into its first writer.
  std::set<int> observable = pinned;
  for (auto& g : P.grads) observable.insert(g.second);
  if (P.loss >= 0) observable.insert(P.loss);
  for (int i = nO - 1; i >= 0; --i) {
    if (op_done_[i] || P.kind[i] != "permute") continue;
    int a = P.op(i)["a"].i32(), o = P.out[i];
    const TView& va = views_[a];
    if (va.root != a || !va.contiguous || va.onehot || observable.count(a)) continue;
    if (P.consumers[a].size() != 1 || P.consumers[a][0] != i) continue;
    int p = P.producer[a];
    if (p < 0 || op_done_[p] || action_[p] != 0) continue;
    const bool gemm_writer = is_gemm(p) && P.T[a].shape.size() <= 4;
    const bool perm_writer = P.kind[p] == "permute";
    if (!gemm_writer && !perm_writer) continue;
    const TView& vo = views_[o];
    if (vo.onehot) continue;
    const auto& perm = P.op(i)["perm"].a;
    TView nv;
    nv.root = vo.root;
    nv.off = vo.off;
    nv.strides.assign(perm.size(), 0);
    for (size_t d = 0; d < perm.size(); ++d) nv.strides[perm[d].i32()] = vo.strides[d];
    nv.contiguous = nv.strides == contig_strides(P.T[a].shape);
    views_[a] = nv;
    op_done_[i] = 1;
  }

  plan_attention(observable);

  // A scale whose input only a GEMM writes and nothing else reads becomes
  // that GEMM's alpha: the GEMM stores alpha * acc, rounded once as the
  // mul_scalar would, straight into the scaled tensor's storage (attention's
  // 1/sqrt(d) on the scores).
  for (int i = 0; i < nO; ++i) {
    if (op_done_[i] || P.kind[i] != "mul_scalar") continue;
    int a = P.op(i)["a"].i32(), o = P.out[i];
    int p = P.producer[a];
    if (p < 0 || !is_gemm(p) || op_done_[p] || action_[p] != 0 || gemm_alpha_[p] != 1.f) continue;
    if (observable.count(a) || P.consumers[a].size() != 1 || P.T[a].shape != P.T[o].shape) continue;
    const TView& va = views_[a];
    const TView& vo = views_[o];
    if (va.root != a || !va.contiguous || va.onehot || vo.onehot || !vo.contiguous) continue;
    views_[a] = vo;
    gemm_alpha_[p] = (float)P.op(i)["scalar"].num();
    op_done_[i] = 1;
  }
}

// ------------------------------------------------------------ optimizer ----
void Graph::plan_optimizer() {
  if (parent) return;
  std::map<std::string, int> param_t, grad_t, state_t;
  for (auto& p : P.params) param_t[p.first] = p.second;
  for (auto& g : P.grads) grad_t[g.first] = g.second;
  for (auto& s : P.states) state_t[s.name] = s.tensor;
  std::map<std::string, int> wb_src;
  for (auto& w : P.writebacks) wb_src[(w.to_param ? "p:" : "s:") + w.dest] = w.src;
  auto only_consumer = [&](int t, int op) {
    return P.consumers[t].size() == 1 && P.consumers[t][0] == op;
  };
  const std::string okind = P.optimizer ? (*P.optimizer)["kind"].str() : std::string();
  std::vector<std::pair<std::string, bool>> decayed;  // name, decayed
  std::vector<int> fold;

  if (okind == "adam") {
    int lrt = -1, shrink_t = -1;
    float shrink_lit = 1.f, b1 = 0, b2 = 0, eps = 0;
    bool ok = !P.grads.empty();
    for (auto& pg : P.grads) {
      if (!ok) break;
      const std::string& n = pg.first;
      auto ip = wb_src.find("p:" + n), im = wb_src.find("s:adam_m_" + n), iv = wb_src.find("s:adam_v_" + n);
      if (ip == wb_src.end() || im == wb_src.end() || iv == wb_src.end()) { ok = false; break; }
      int op_p = P.producer[ip->second], op_m = P.producer[im->second], op_v = P.producer[iv->second];
      if (P.kind[op_p] != "adam_update_p" || P.kind[op_m] != "adam_update_m" || P.kind[op_v] != "adam_update_v") {
        ok = false; break;
      }
      const auto& OP = P.op(op_p); const auto& OM = P.op(op_m); const auto& OV = P.op(op_v);
      int G = pg.second;
      if (OP["p"].i32() != param_t[n] || OP["mNew"].i32() != P.out[op_m] || OP["vNew"].i32() != P.out[op_v] ||
          OM["g"].i32() != G || OV["g"].i32() != G || OM["m"].i32() != state_t["adam_m_" + n] ||
          OV["v"].i32() != state_t["adam_v_" + n] || !only_consumer(P.out[op_m], op_p) ||
          !only_consumer(P.out[op_v], op_p) || !P.consumers[P.out[op_p]].empty()) {
        ok = false; break;
      }
      if (lrt < 0) { lrt = OP["lrt"].i32(); b1 = (float)OM["beta1"].num(); b2 = (float)OV["beta2"].num();
                     eps = (float)OP["eps"].num(); }
      if (OP["lrt"].i32() != lrt || (float)OM["beta1"].num() != b1 || (float)OV["beta2"].num() != b2 ||
          (float)OP["eps"].num() != eps) { ok = false; break; }
      bool dec;
      if (!OP["decayShrinkTensor"].is_null()) {
        int st = OP["decayShrinkTensor"].i32();
        if (shrink_t >= 0 && shrink_t != st) { ok = false; break; }
        shrink_t = st; dec = true;
      } else {
        float lit = (float)OP["decayShrink"].num();
        dec = lit != 1.0f;
        if (dec) {
          if (shrink_lit != 1.0f && shrink_lit != lit) { ok = false; break; }
          shrink_lit = lit;
        }
      }
      decayed.emplace_back(n, dec);
      fold.push_back(op_p); fold.push_back(op_m); fold.push_back(op_v);
    }
    if (shrink_t >= 0 && shrink_lit != 1.0f) ok = false;
    if (ok) {
      adam_fused_ = true;
      adam_lrt_ = lrt;
      adam_shrink_ = shrink_t;
      const double b1d = (*P.optimizer)["config"]["beta1"].num(), b2d = (*P.optimizer)["config"]["beta2"].num();
      adam_.beta1 = (float)b1d; adam_.one_minus_beta1 = (float)(1.0 - b1d);
      adam_.beta2 = (float)b2d; adam_.one_minus_beta2 = (float)(1.0 - b2d);
      adam_.eps = eps;
      adam_.shrink_lit = shrink_lit;
    }
  } else if (okind == "sgd") {
    // p_new = sub(p, mul(broadcast_to(lr), upd)); upd = v_new | add(g_eff, mul_scalar(v_new, mu)) | g_eff
    // v_new = add(mul_scalar(v, mu), g_eff); g_eff = G | add(G, mul_scalar(p, wd))
    const auto& cfg = (*P.optimizer)["config"];
    double mu = cfg["momentum"].num(), wd = cfg["weightDecay"].num();
    bool nesterov = cfg["nesterov"].kind == tgjson::Value::Bool && cfg["nesterov"].b;
    int lr_t = -1;
    bool ok = !P.grads.empty();
    for (auto& pg : P.grads) {
      if (!ok) break;
      const std::string& n = pg.first;
      int G = pg.second, pt = param_t[n];
      auto ip = wb_src.find("p:" + n);
      if (ip == wb_src.end()) { ok = false; break; }
      int o_sub = P.producer[ip->second];
      if (P.kind[o_sub] != "sub" || P.op(o_sub)["a"].i32() != pt) { ok = false; break; }
      int o_mul = P.producer[P.op(o_sub)["b"].i32()];
      if (P.kind[o_mul] != "mul") { ok = false; break; }
      int o_bc = P.producer[P.op(o_mul)["a"].i32()];
      if (P.kind[o_bc] != "broadcast_to") { ok = false; break; }
      int lr_here = P.op(o_bc)["a"].i32();
      if (lr_t >= 0 && lr_here != lr_t) { ok = false; break; }
      lr_t = lr_here;
      int upd = P.op(o_mul)["b"].i32();
      std::vector<int> f = {o_sub, o_mul, o_bc};
      int g_eff = -1;
      if (mu > 0) {
        auto iv = wb_src.find("s:sgd_v_" + n);
        if (iv == wb_src.end()) { ok = false; break; }
        int vnew = iv->second;
        int o_vadd = P.producer[vnew];
        if (P.kind[o_vadd] != "add") { ok = false; break; }
        int o_vms = P.producer[P.op(o_vadd)["a"].i32()];
        if (P.kind[o_vms] != "mul_scalar" || P.op(o_vms)["a"].i32() != state_t["sgd_v_" + n]) { ok = false; break; }
        g_eff = P.op(o_vadd)["b"].i32();
        f.push_back(o_vadd); f.push_back(o_vms);
        if (nesterov) {
          int o_nadd = P.producer[upd];
          if (P.kind[o_nadd] != "add" || P.op(o_nadd)["a"].i32() != g_eff) { ok = false; break; }
          int o_nms = P.producer[P.op(o_nadd)["b"].i32()];
          if (P.kind[o_nms] != "mul_scalar" || P.op(o_nms)["a"].i32() != vnew) { ok = false; break; }
          f.push_back(o_nadd); f.push_back(o_nms);
        } else if (upd != vnew) { ok = false; break; }
      } else {
        g_eff = upd;
      }
      bool dec = false;
      if (g_eff != G) {
        int o_gadd = P.producer[g_eff];
        if (o_gadd < 0 || P.kind[o_gadd] != "add" || P.op(o_gadd)["a"].i32() != G) { ok = false; break; }
        int o_gms = P.producer[P.op(o_gadd)["b"].i32()];
        if (P.kind[o_gms] != "mul_scalar" || P.op(o_gms)["a"].i32() != pt) { ok = false; break; }
        f.push_back(o_gadd); f.push_back(o_gms);
        dec = true;
      }
      decayed.emplace_back(n, dec);
      for (int x : f) fold.push_back(x);
    }
    if (ok) {
      sgd_fused_ = true;
      sgd_lr_ = lr_t;
      sgd_.momentum = (float)mu;
      sgd_.wd = (float)wd;
      sgd_.nesterov = nesterov ? 1 : 0;
    }
  }
  // Flat layout: decayed params first so one index split selects the shrink.
  std::vector<std::string> order;
  if (adam_fused_ || sgd_fused_) {
    for (auto& d : decayed) if (d.second) order.push_back(d.first);
    for (auto& d : decayed) if (!d.second) order.push_back(d.first);
    for (int x : fold) op_done_[x] = 1;
  }
  for (auto& p : P.params)
    if (std::find(order.begin(), order.end(), p.first) == order.end()) order.push_back(p.first);
  int64_t off = 0;
  n_decay_ = 0;
  for (auto& n : order) {
    int64_t numel = P.T[param_t[n]].numel;
    bool dec = false;
    for (auto& d : decayed) if (d.first == n) dec = d.second;
    layout_.emplace_back(n, (int)numel);
    param_off_[n] = off * 4;
    param_n_[n] = numel;
    off += (numel + 63) / 64 * 64;
    if (dec) n_decay_ = off;
  }
  flat_floats_ = off;
}

}  // namespace tg

namespace tg {

// Causal attention blocks, matched on the op chain the tracer and autodiff
// emit (src/ops.ts softmaxCausal and dropout, src/grad.ts rules for matmul,
// softmaxCausal, dropout and mulScalar):
//
//   s = matmul_batched(q, permute(k, swap)), s2 = mul_scalar(s, c),
//   p = softmax_causal_last(s2), pd = dropout(p) (optional), o = matmul_batched(pd, v)
//
// and, when the graph trains, the gradient ops
//
//   dpd = matmul_batched(dO, permute(v)), dv = matmul_batched(permute(pd), dO),
//   dp = dropout(dpd) (same p and salt), r = sum_last(mul(dp, p)),
//   ds = mul_scalar(mul(sub(dp, broadcast(reshape(r))), p), c),
//   dq = matmul_batched(ds, permute(permute(k))), dkt = matmul_batched(permute(q), ds).
//
// Every intermediate (s, s2, p, pd, dpd, dp, ...) must be read by exactly
// these ops and be unobservable (not captured, not an output); otherwise the
// block runs unfused. Head dims 16, 32 and 64 are fused.
//
// The fused kernels never materialise the [B, H, T, T] scores and
// probabilities; measured on B200 they take about the time of the unfused
// chain (tensor-core GEMMs plus memory-bound passes) at T = 1024 and longer
// below it. So by default a block is fused when one probabilities tensor
// would take at least 1 GiB; TG_ATTN_FUSE=1 fuses every matching block,
// TG_ATTN_FUSE=0 none.
void Graph::plan_attention(const std::set<int>& observable) {
  const char* env = getenv("TG_ATTN_FUSE");
  const int mode = env && env[0] == '1' ? 1 : (env && env[0] == '0' ? 0 : -1);
  if (mode == 0) return;
  const int nO = (int)P.ops.size();
  auto kind_is = [&](int op, const char* k) { return op >= 0 && P.kind[op] == k; };
  auto only = [&](int t, std::initializer_list<int> ops) {
    if (observable.count(t)) return false;
    std::set<int> want(ops), got(P.consumers[t].begin(), P.consumers[t].end());
    return want == got && P.consumers[t].size() == want.size();
  };
  auto swap_perm = [&](int op) {
    if (!kind_is(op, "permute")) return false;
    const auto& pv = P.op(op)["perm"].a;
    return pv.size() == 4 && pv[0].i32() == 0 && pv[1].i32() == 1 && pv[2].i32() == 3 && pv[3].i32() == 2;
  };
  auto in = [&](int op, const char* f) { return P.op(op)[f].i32(); };
  auto rank4 = [&](int t) { return P.T[t].shape.size() == 4 && !views_[t].onehot; };
  auto consumer_of_kind = [&](int t, const char* k) {
    for (int c : P.consumers[t]) if (kind_is(c, k)) return c;
    return -1;
  };

  for (int f5 = 0; f5 < nO; ++f5) {
    if (op_done_[f5] || action_[f5] != 0 || !kind_is(f5, "matmul_batched")) continue;
    const int pd = in(f5, "a"), v = in(f5, "b"), o = P.out[f5];
    if (!rank4(pd) || !rank4(v) || !rank4(o)) continue;
    int f4 = P.producer[pd], p_t = pd;
    const bool drop = kind_is(f4, "dropout");
    if (drop) p_t = in(f4, "a");
    const int f3 = P.producer[p_t];
    if (!kind_is(f3, "softmax_causal_last")) continue;
    const int s2 = in(f3, "a"), f2 = P.producer[s2];
    if (!kind_is(f2, "mul_scalar") || !only(s2, {f3})) continue;
    const int s = in(f2, "a"), f1 = P.producer[s];
    if (!kind_is(f1, "matmul_batched") || !only(s, {f2}) || op_done_[f1]) continue;
    const int q = in(f1, "a"), kt = in(f1, "b");
    const int fk = P.producer[kt];
    if (!swap_perm(fk) || !rank4(q)) continue;
    const int k = in(fk, "a");
    const auto& qs = P.T[q].shape;
    const int64_t Bn = qs[0], Hn = qs[1], Tn = qs[2], Dn = qs[3];
    if (!attn_supported_dim((int)Dn) || P.T[k].shape != qs || P.T[v].shape != qs) continue;
    if (P.T[p_t].shape != std::vector<int64_t>{Bn, Hn, Tn, Tn}) continue;
    if (mode < 0 && P.T[p_t].numel * 4 < ((int64_t)1 << 30)) continue;
    const float scale = (float)P.op(f2)["scalar"].num();

    AttnBlock A{};
    A.q = q; A.k = k; A.kt = kt; A.v = v; A.o = o;
    A.dout = A.dv = A.ds = A.dq = A.dkt = -1;
    A.ml = s; A.p_t = p_t; A.scale = scale; A.dropout = drop;
    A.p = drop ? f32_lit8(P.op(f4)["p"].num()) : 0.f;
    A.keep_scale = drop ? f32_lit8(1.0 / (1.0 - P.op(f4)["p"].num())) : 1.f;
    A.salt = drop ? (uint32_t)(((uint64_t)P.op(f4)["salt"].i64() * 0x9E3779B1ull) & 0xFFFFFFFFull) : 0u;
    std::vector<int> done = {f1, f2, f3};
    if (drop) done.push_back(f4);

    // backward, if the probabilities are read beyond the forward
    const bool fwd_only = drop ? (only(p_t, {f4}) && only(pd, {f5})) : only(p_t, {f5});
    int bwd = -1;
    if (!fwd_only) {
      bool ok = true;
      // dv = matmul_batched(permute(pd), dO)
      int pdt_op = -1;
      for (int c : P.consumers[pd]) if (c != f5 && swap_perm(c)) pdt_op = c;
      ok = ok && swap_perm(pdt_op) && (drop ? only(pd, {f5, pdt_op}) : true);
      const int pdt = ok ? P.out[pdt_op] : -1;
      const int bdv = ok ? consumer_of_kind(pdt, "matmul_batched") : -1;
      ok = ok && bdv >= 0 && only(pdt, {bdv}) && in(bdv, "a") == pdt;
      const int dO = ok ? in(bdv, "b") : -1;
      // dpd = matmul_batched(dO, permute(v))
      int bdp = -1;
      if (ok)
        for (int c : P.consumers[dO])
          if (kind_is(c, "matmul_batched") && in(c, "a") == dO && swap_perm(P.producer[in(c, "b")]) &&
              in(P.producer[in(c, "b")], "a") == v)
            bdp = c;
      ok = ok && bdp >= 0;
      const int dpd = ok ? P.out[bdp] : -1;
      int dp = dpd, bdrop = -1;
      if (ok && drop) {
        bdrop = consumer_of_kind(dpd, "dropout");
        ok = bdrop >= 0 && only(dpd, {bdrop}) && P.op(bdrop)["salt"].i64() == P.op(f4)["salt"].i64() &&
             P.op(bdrop)["p"].num() == P.op(f4)["p"].num();
        dp = ok ? P.out[bdrop] : -1;
      }
      // r = sum_last(mul(dp, p)); ds = mul_scalar(mul(sub(dp, broadcast(reshape(r))), p), c)
      int m1 = -1, sb = -1;
      if (ok)
        for (int c : P.consumers[dp]) {
          if (kind_is(c, "mul")) m1 = c;
          if (kind_is(c, "sub") && in(c, "a") == dp) sb = c;
        }
      ok = ok && m1 >= 0 && sb >= 0 && only(dp, {m1, sb});
      ok = ok && ((in(m1, "a") == dp && in(m1, "b") == p_t) || (in(m1, "b") == dp && in(m1, "a") == p_t));
      const int rs = ok ? consumer_of_kind(P.out[m1], "sum_last") : -1;
      ok = ok && rs >= 0 && only(P.out[m1], {rs});
      const int rr = ok ? consumer_of_kind(P.out[rs], "reshape") : -1;
      ok = ok && rr >= 0 && only(P.out[rs], {rr});
      const int rb = ok ? consumer_of_kind(P.out[rr], "broadcast_to") : -1;
      ok = ok && rb >= 0 && only(P.out[rr], {rb}) && only(P.out[rb], {sb}) && in(sb, "b") == P.out[rb];
      const int m2 = ok ? consumer_of_kind(P.out[sb], "mul") : -1;
      ok = ok && m2 >= 0 && only(P.out[sb], {m2}) &&
           ((in(m2, "a") == P.out[sb] && in(m2, "b") == p_t) || (in(m2, "b") == P.out[sb] && in(m2, "a") == p_t));
      const int ms = ok ? consumer_of_kind(P.out[m2], "mul_scalar") : -1;
      ok = ok && ms >= 0 && only(P.out[m2], {ms}) && (float)P.op(ms)["scalar"].num() == scale;
      const int ds = ok ? P.out[ms] : -1;
      // dq = matmul_batched(ds, permute(kt)), dkt = matmul_batched(permute(q), ds)
      int bdq = -1, bdk = -1;
      if (ok)
        for (int c : P.consumers[ds]) {
          if (!kind_is(c, "matmul_batched")) continue;
          if (in(c, "a") == ds && swap_perm(P.producer[in(c, "b")]) && in(P.producer[in(c, "b")], "a") == kt) bdq = c;
          if (in(c, "b") == ds && swap_perm(P.producer[in(c, "a")]) && in(P.producer[in(c, "a")], "a") == q) bdk = c;
        }
      ok = ok && bdq >= 0 && bdk >= 0 && only(ds, {bdq, bdk});
      ok = ok && (drop ? only(p_t, {f4, m1, m2}) : only(p_t, {f5, pdt_op, m1, m2}));
      // dS is written as full [B, H, T, T] rows
      ok = ok && views_[ds].root == ds && views_[ds].contiguous && views_[ds].off == 0;
      ok = ok && rank4(dO) && rank4(P.out[bdv]) && rank4(P.out[bdq]) && rank4(P.out[bdk]);
      if (!ok) continue;
      A.dout = dO; A.dv = P.out[bdv]; A.ds = ds; A.dq = P.out[bdq]; A.dkt = P.out[bdk];
      A.rowdot = P.out[rs];
      for (int x : {bdv, m1, rs, rr, rb, sb, m2, ms, bdk}) done.push_back(x);
      if (drop) done.push_back(bdrop);
      bwd = std::min({bdp, bdv, bdk});
      for (int x : {bdp, bdq}) if (x != bwd) done.push_back(x);
    }
    // commit
    const int id = (int)attn_.size();
    attn_.push_back(A);
    for (int x : done) if (x != bwd) op_done_[x] = 1;
    action_[f5] = 110;
    attn_of_[f5] = id;
    fused_io_[f5] = {{q, k, v}, {o, s}};
    bytes_override_[s] = 2 * Bn * Hn * Tn * 4;
    if (bwd >= 0) {
      op_done_[bwd] = 0;
      action_[bwd] = 111;
      attn_of_[bwd] = id;
      fused_io_[bwd] = {{q, k, v, o, A.dout, s}, {A.dv, A.ds, A.dkt, A.dq, A.rowdot}};
    }
  }
}

}  // namespace tg

namespace tg {
std::vector<int> Graph::eff_consumers(int t) const {
  std::vector<int> out;
  for (int c : P.consumers[t])
    if (!no_read_.count({c, t})) out.push_back(c);
  return out;
}
}  // namespace tg
