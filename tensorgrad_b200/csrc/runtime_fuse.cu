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

constexpr int kMaxGroupInputs = 12;
constexpr int kMaxGroupOps = 48;

}  // namespace

bool Graph::ew_internal(int t) const {
  if (ew_root_.empty()) return false;
  int p = P.producer[t];
  return p >= 0 && ew_root_[p] >= 0 && ew_root_[p] != p;
}

void Graph::plan_fusion() {
  const int nO = (int)P.ops.size();
  ew_root_.assign(nO, -1);
  jit_ = jit_enabled();
  if (!jit_) return;
  std::set<int> observable;
  for (int t : P.outputs) observable.insert(t);
  for (auto& c : P.captures) observable.insert(c.second);
  for (auto& w : P.writebacks) observable.insert(w.src);
  for (auto& g : P.grads) observable.insert(g.second);
  if (P.loss >= 0) observable.insert(P.loss);
  for (int i = 0; i < nO; ++i)
    if (!op_done_[i] && action_[i] == 0 && ew_kinds().count(P.kind[i])) ew_root_[i] = i;

  std::vector<std::vector<int>> members(nO);
  std::vector<std::set<int>> ext(nO);  // tensors a group reads from memory
  std::vector<char> posdep(nO, 0);     // group uses the element index (dropout, causal mask)
  for (int i = 0; i < nO; ++i) posdep[i] = P.kind[i] == "dropout" || P.kind[i] == "where_causal";
  auto side = [&](int i) { return P.opt_start >= 0 && i >= P.opt_start; };
  for (int i = 0; i < nO; ++i) {
    if (ew_root_[i] != i) continue;
    members[i] = {i};
    for (int t : ew_operands(P, i)) ext[i].insert(t);
    std::vector<int> ops_in = ew_operands(P, i);
    std::set<int> seen;
    for (int t : ops_in) {
      if (!seen.insert(t).second) continue;
      int p = P.producer[t];
      if (p < 0 || ew_root_[p] != p || members[p].empty()) continue;
      if (P.consumers[t].size() != 1 || P.consumers[t][0] != i) continue;
      if (observable.count(t)) continue;
      const TView& v = views_[t];
      if (v.root != t || v.onehot || !v.contiguous) continue;
      if (P.T[t].shape != P.T[P.out[i]].shape) {
        // a smaller producer whose value the consumer reads broadcast is
        // recomputed per output element; exact for pure elementwise ops, but
        // not for ones that use the element's position
        if (!broadcasts_to(P.T[t].shape, P.T[P.out[i]].shape) || posdep[p]) continue;
      }
      if (side(p) != side(i)) continue;
      std::set<int> merged = ext[i];
      merged.erase(t);
      merged.insert(ext[p].begin(), ext[p].end());
      if ((int)merged.size() > kMaxGroupInputs) continue;
      if ((int)(members[i].size() + members[p].size()) > kMaxGroupOps) continue;
      posdep[i] = posdep[i] || posdep[p];
      for (int m : members[p]) ew_root_[m] = i;
      members[i].insert(members[i].end(), members[p].begin(), members[p].end());
      members[p].clear();
      ext[p].clear();
      ext[i] = std::move(merged);
    }
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

void Graph::emit_ew_group(int r, const int* seed_ptr,
                          const std::function<void(const std::string&, std::function<void(cudaStream_t)>)>& add) {
  std::vector<int> mem;
  for (int m = 0; m <= r; ++m)
    if (ew_root_[m] == r) mem.push_back(m);
  const int o = P.out[r];
  const auto& os = P.T[o].shape;
  const int64_t n = P.T[o].numel;
  if (n <= 0) return;
  bool vec = true;
  std::vector<EwInput> ins;
  std::vector<int> in_t;
  std::map<int, int> slot_of;
  bool has_drop = false;
  std::ostringstream ops;
  std::string label;
  for (int m : mem) {
    std::vector<std::string> a;
    for (int t : ew_operands(P, m)) {
      if (ew_internal(t) && ew_root_[P.producer[t]] == r) { a.push_back("v" + std::to_string(t)); continue; }
      auto it = slot_of.find(t);
      if (it == slot_of.end()) {
        it = slot_of.emplace(t, (int)ins.size()).first;
        ins.push_back(ew_input(t, os, vec));
        in_t.push_back(t);
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
  void* out = ptr(o);
  vec = vec && n % 4 == 0 && ((uintptr_t)out & 15) == 0;
  const int R = (int)os.size();

  // Per-lane values of each input (and, for the vector form, the loads that
  // precede the lane loop).
  std::ostringstream pre, lane;
  for (size_t s = 0; s < ins.size(); ++s) {
    const EwInput& in = ins[s];
    std::string p = "p" + std::to_string(s), x = "x" + std::to_string(s);
    std::string per = std::to_string(in.period) + "ll";
    switch (in.mode) {
      case IN_FULL:
        if (vec) { pre << "    const float4 q" << s << " = __ldg(reinterpret_cast<const float4*>(" << p << " + i));\n";
                   lane << "      const float " << x << " = f4(q" << s << ", l);\n"; }
        else lane << "      const float " << x << " = __ldg(" << p << " + e);\n";
        break;
      case IN_SCALAR:
        pre << "    const float s" << s << " = __ldg(" << p << ");\n";
        lane << "      const float " << x << " = s" << s << ";\n";
        break;
      case IN_PERIOD:
        if (vec) { pre << "    const float4 q" << s << " = __ldg(reinterpret_cast<const float4*>(" << p << " + i % " << per << "));\n";
                   lane << "      const float " << x << " = f4(q" << s << ", l);\n"; }
        else lane << "      const float " << x << " = __ldg(" << p << " + e % " << per << ");\n";
        break;
      case IN_ROWDIV:
        if (vec) { pre << "    const float s" << s << " = __ldg(" << p << " + i / " << per << ");\n";
                   lane << "      const float " << x << " = s" << s << ";\n"; }
        else lane << "      const float " << x << " = __ldg(" << p << " + e / " << per << ");\n";
        break;
      case IN_ONEHOT:
        lane << "      const float " << x << " = ((i64)__ldg(reinterpret_cast<const int*>(" << p << ") + e / " << per
             << ") == e % " << per << ") ? 1.f : 0.f;\n";
        break;
      default: {  // IN_STRIDED: row-major coordinates of e, dotted with the operand's strides
        lane << "      i64 o" << s << " = 0;\n      { i64 rem = e;\n";
        for (int d = R - 1; d >= 0; --d) {
          if (os[d] == 1) continue;
          if (in.strides[d] != 0)
            lane << "        o" << s << " += (rem % " << os[d] << "ll) * " << in.strides[d] << "ll;\n";
          if (d > 0) lane << "        rem /= " << os[d] << "ll;\n";
        }
        lane << "      }\n      const float " << x << " = __ldg(" << p << " + o" << s << ");\n";
      }
    }
  }

  std::ostringstream k;
  k << "(";
  for (size_t s = 0; s < ins.size(); ++s) k << "const float* __restrict__ p" << s << ", ";
  k << "float* __restrict__ out, const int* __restrict__ seedp, i64 drop_off) {\n";
  k << "  const u32 seed = " << (has_drop ? "seedp ? (u32)(*seedp) : 0u" : "0u") << ";\n";
  k << "  (void)seed; (void)drop_off;\n";
  if (vec) {
    k << "  for (i64 t = (i64)blockIdx.x * 256 + threadIdx.x; t < " << n / 4 << "ll; t += (i64)gridDim.x * 256) {\n";
    k << "    const i64 i = t * 4;\n" << pre.str();
    k << "    float r[4];\n#pragma unroll\n    for (int l = 0; l < 4; ++l) {\n      const i64 e = i + l;\n";
    k << lane.str() << ops.str() << "      r[l] = v" << o << ";\n    }\n";
    k << "    *reinterpret_cast<float4*>(out + i) = make_float4(r[0], r[1], r[2], r[3]);\n  }\n}\n";
  } else {
    k << "  for (i64 e = (i64)blockIdx.x * 256 + threadIdx.x; e < " << n << "ll; e += (i64)gridDim.x * 256) {\n";
    k << pre.str() << lane.str() << ops.str() << "      out[e] = v" << o << ";\n  }\n}\n";
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
    const int* seed;
    long long drop_off;
  };
  auto A = std::make_shared<Args>();
  for (auto& in : ins) A->in.push_back(in.ptr);
  A->out = out;
  A->seed = seed_ptr;
  A->drop_off = (long long)ctx->rank * n;
  const int64_t work = vec ? n / 4 : n;
  int64_t blocks = (work + 255) / 256, cap = (int64_t)device_sm_count() * 8;
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min(blocks, cap));
  if (mem.size() > 1) label = "fused_ew|" + label.substr(0, 160);
  add(label, [fn, A, grid](cudaStream_t s) {
    std::vector<void*> args;
    for (auto& p : A->in) args.push_back(const_cast<const void**>(&p));
    args.push_back(&A->out);
    args.push_back(const_cast<const int**>(&A->seed));
    args.push_back(&A->drop_off);
    jit_launch(*fn, grid, 256, args.data(), s);
  });
}

}  // namespace tg
