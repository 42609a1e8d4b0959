// extern "C" entry points of libtgcuda.so (declared in include/tensorgrad_b200.h).
#include <nccl.h>

#include <cstring>
#include <string>

#include "../../include/tensorgrad_b200.h"
#include "runtime.hpp"

struct tg_ctx {
  tg::Context* c;
};

namespace {
thread_local std::string g_err_name = "";
thread_local std::string g_err_msg = "";

int fail(const std::string& name, const std::string& msg) {
  g_err_name = name;
  g_err_msg = msg;
  if (name == "AbortError") return TG_ABORTED;
  if (name == "CudaError") return TG_CUDA_ERR;
  if (name == "NcclError") return TG_NCCL_ERR;
  return TG_ERR;
}

template <typename F>
int guarded(F&& f) {
  try {
    f();
    g_err_name.clear();
    g_err_msg.clear();
    return TG_OK;
  } catch (const tg::TgError& e) {
    return fail(e.name, e.what());
  } catch (const std::exception& e) {
    return fail("Error", e.what());
  } catch (...) {
    return fail("Error", "unknown failure");
  }
}

tg::Graph* get_graph(tg_ctx* ctx, int gid) {
  if (!ctx || !ctx->c) throw tg::TgError("Error", "null context");
  auto it = ctx->c->graphs.find(gid);
  if (it == ctx->c->graphs.end()) throw tg::TgError("AbortError", "graph " + std::to_string(gid) + " does not exist (destroyed or replaced)");
  cudaSetDevice(ctx->c->device);
  return it->second.get();
}

void write_str(const std::string& s, char* buf, size_t cap, size_t* needed) {
  if (needed) *needed = s.size() + 1;
  if (buf && cap > 0) {
    size_t n = s.size() < cap - 1 ? s.size() : cap - 1;
    memcpy(buf, s.data(), n);
    buf[n] = 0;
  }
}
}  // namespace

namespace tg {
int api_fail(const std::string& name, const std::string& msg) { return fail(name, msg); }
int api_ok() {
  g_err_name.clear();
  g_err_msg.clear();
  return TG_OK;
}
}  // namespace tg

extern "C" {

int tg_nccl_unique_id(uint8_t out[128]) {
  return guarded([&] {
    ncclUniqueId id;
    ncclResult_t r = ncclGetUniqueId(&id);
    if (r != ncclSuccess) throw tg::TgError("NcclError", ncclGetErrorString(r));
    static_assert(sizeof(id) == 128, "nccl id size");
    memcpy(out, &id, 128);
  });
}

int tg_ctx_create(int device, int rank, int world, const uint8_t* nccl_id, tg_ctx** out) {
  return guarded([&] {
    *out = nullptr;
    auto* c = new tg::Context(device, rank, world, nccl_id);
    *out = new tg_ctx{c};
  });
}

int tg_ctx_destroy(tg_ctx* ctx) {
  return guarded([&] {
    if (!ctx) return;
    if (ctx->c) {
      cudaSetDevice(ctx->c->device);
      cudaStreamSynchronize(ctx->c->stream);
      delete ctx->c;
    }
    delete ctx;
  });
}

int tg_graph_create(tg_ctx* ctx, int graph_id, int parent_graph_id, const char* program_json, size_t len) {
  return guarded([&] {
    if (!ctx || !ctx->c) throw tg::TgError("Error", "null context");
    cudaSetDevice(ctx->c->device);
    tg::Graph* parent = nullptr;
    if (parent_graph_id >= 0) parent = get_graph(ctx, parent_graph_id);
    ctx->c->graphs.erase(graph_id);
    auto g = std::make_unique<tg::Graph>(ctx->c, graph_id, parent, program_json, len);
    ctx->c->graphs[graph_id] = std::move(g);
  });
}

int tg_graph_info(tg_ctx* ctx, int graph_id, char* buf, size_t cap, size_t* needed) {
  return guarded([&] { write_str(get_graph(ctx, graph_id)->info_json(), buf, cap, needed); });
}

int tg_plan_dry(const char* program_json, size_t len, int world, char* buf, size_t cap, size_t* needed) {
  return guarded([&] {
    if (world < 1) throw tg::TgError("Error", "tg_plan_dry: world must be >= 1");
    tg::Context c(tg::Context::Dry{}, world);
    tg::Graph g(&c, 0, nullptr, program_json, len);
    std::string s = "{\"info\":" + g.info_json() + ",\"launches\":[";
    auto q = [](const std::string& x) {
      std::string o = "\"";
      for (char ch : x) {
        if (ch == '"' || ch == '\\') { o += '\\'; o += ch; }
        else if (ch == '\n') o += "\\n";
        else o += ch;
      }
      return o + "\"";
    };
    std::string kinds = g.launch_kinds();
    size_t st = 0;
    bool first = true;
    for (size_t e; (e = kinds.find('\n', st)) != std::string::npos; st = e + 1) {
      if (!first) s += ",";
      first = false;
      s += q(kinds.substr(st, e - st));
    }
    s += "],\"launchBytes\":[";
    for (size_t i = 0; i < g.launch_bytes().size(); ++i) s += (i ? "," : "") + std::to_string(g.launch_bytes()[i]);
    s += "],\"kernelSources\":[";
    for (size_t i = 0; i < g.jit_sources().size(); ++i) s += (i ? "," : "") + q(g.jit_sources()[i]);
    s += "],\"kernelPreamble\":" + q(tg::jit_preamble()) + "}";
    write_str(s, buf, cap, needed);
  });
}

int tg_launch_list(tg_ctx* ctx, int graph_id, char* buf, size_t cap, size_t* needed) {
  return guarded([&] { write_str(get_graph(ctx, graph_id)->launch_kinds(), buf, cap, needed); });
}

int tg_upload_params(tg_ctx* ctx, int graph_id, int n, const char* const* names, const float* const* data,
                     const size_t* numel) {
  return guarded([&] { get_graph(ctx, graph_id)->upload_params(n, names, data, numel); });
}

int tg_download_params(tg_ctx* ctx, int graph_id, int n, const char* const* names, float* const* out,
                       const size_t* numel) {
  return guarded([&] { get_graph(ctx, graph_id)->download_params(n, names, out, numel); });
}

int tg_upload_states(tg_ctx* ctx, int graph_id, int n, const char* const* names, const float* const* data,
                     const size_t* numel) {
  return guarded([&] { get_graph(ctx, graph_id)->upload_states(n, names, data, numel); });
}

int tg_download_states(tg_ctx* ctx, int graph_id, int n, const char* const* names, float* const* out,
                       const size_t* numel) {
  return guarded([&] { get_graph(ctx, graph_id)->download_states(n, names, out, numel); });
}

int tg_get_counters(tg_ctx* ctx, int graph_id, int64_t* step, int64_t* prng) {
  return guarded([&] {
    if (!step || !prng) throw tg::TgError("Error", "tg_get_counters: null output");
    get_graph(ctx, graph_id)->get_counters(step, prng);
  });
}

int tg_set_counters(tg_ctx* ctx, int graph_id, int64_t step, int64_t prng) {
  return guarded([&] {
    if (step < 0 || prng < 0) throw tg::TgError("Error", "tg_set_counters: negative counter");
    get_graph(ctx, graph_id)->set_counters(step, prng);
  });
}

int tg_step(tg_ctx* ctx, int graph_id, int n, const char* const* names, const void* const* data,
            const size_t* bytes, float* loss_out, void* const* capture_out) {
  return guarded([&] {
    tg::Graph* g = get_graph(ctx, graph_id);
    g->require_inputs(n, names);
    g->set_inputs(n, names, data, bytes, false);
    g->launch_step();
    g->read_loss(loss_out);
    if (capture_out) g->read_captures(capture_out);
  });
}

int tg_run(tg_ctx* ctx, int graph_id, int n, const char* const* names, const void* const* data,
           const size_t* bytes, void* output_out, void* const* capture_out) {
  return guarded([&] {
    tg::Graph* g = get_graph(ctx, graph_id);
    g->require_inputs(n, names);
    g->set_inputs(n, names, data, bytes, false);
    g->launch_step();
    g->read_output(output_out);
    if (capture_out) g->read_captures(capture_out);
  });
}

int tg_set_inputs(tg_ctx* ctx, int graph_id, int n, const char* const* names, const void* const* data,
                  const size_t* bytes, int device_src) {
  return guarded([&] { get_graph(ctx, graph_id)->set_inputs(n, names, data, bytes, device_src != 0); });
}

int tg_launch_step(tg_ctx* ctx, int graph_id) {
  return guarded([&] { get_graph(ctx, graph_id)->launch_step(); });
}

int tg_read_loss(tg_ctx* ctx, int graph_id, float* loss_out) {
  return guarded([&] { get_graph(ctx, graph_id)->read_loss(loss_out); });
}

int tg_stream(tg_ctx* ctx, void** stream_out) {
  return guarded([&] {
    if (!ctx || !ctx->c) throw tg::TgError("Error", "null context");
    *stream_out = (void*)ctx->c->stream;
  });
}

int tg_reset_optimizer(tg_ctx* ctx, int graph_id) {
  return guarded([&] { get_graph(ctx, graph_id)->reset_optimizer(); });
}

int tg_set_lr(tg_ctx* ctx, int graph_id, const char* lr_json, size_t len) {
  return guarded([&] { get_graph(ctx, graph_id)->set_lr(lr_json, len); });
}

int tg_destroy_graph(tg_ctx* ctx, int graph_id) {
  return guarded([&] {
    if (!ctx || !ctx->c) throw tg::TgError("Error", "null context");
    cudaSetDevice(ctx->c->device);
    cudaStreamSynchronize(ctx->c->stream);
    // destroying a parent cascades to the forward graphs that share its params
    std::vector<int> doomed{graph_id};
    for (auto& kv : ctx->c->graphs)
      if (kv.second->parent && kv.second->parent->id == graph_id) doomed.push_back(kv.first);
    for (int id : doomed) ctx->c->graphs.erase(id);
  });
}

int tg_read_grad(tg_ctx* ctx, int graph_id, const char* name, float* out) {
  return guarded([&] { get_graph(ctx, graph_id)->read_grad(name, out); });
}

int tg_read_tensor(tg_ctx* ctx, int graph_id, int tensor_id, void* out) {
  return guarded([&] { get_graph(ctx, graph_id)->read_tensor(tensor_id, out); });
}

int tg_profile_step(tg_ctx* ctx, int graph_id, float* ms_out, int cap, int* n_out) {
  return guarded([&] {
    std::vector<float> ms;
    get_graph(ctx, graph_id)->profile_step(ms);
    if (n_out) *n_out = (int)ms.size();
    for (int i = 0; i < cap && i < (int)ms.size(); ++i) ms_out[i] = ms[i];
  });
}

int tg_launch_bytes(tg_ctx* ctx, int graph_id, double* out, int cap, int* n_out) {
  return guarded([&] {
    const auto& b = get_graph(ctx, graph_id)->launch_bytes();
    if (n_out) *n_out = (int)b.size();
    for (int i = 0; i < cap && i < (int)b.size(); ++i) out[i] = b[i];
  });
}

int tg_debug_gemm_error(int reset) {
  return tg::gemm_tc_error_flag(reset != 0) | (tg::attn_tc_error_flag(reset != 0) << 8);
}
int tg_debug_gemm_dbg(int* out8) { return tg::gemm_tc_debug(out8); }
int tg_debug_gemm_trace(long long* out, int cap) { return tg::gemm_tc_trace(out, cap); }

const char* tg_last_error_name(void) { return g_err_name.c_str(); }
const char* tg_last_error_message(void) { return g_err_msg.c_str(); }

}  // extern "C"
