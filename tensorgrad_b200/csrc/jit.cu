// Run-time compilation of generated kernels (NVRTC -> sm_100a cubin).
//
// The planner writes one CUDA C kernel per fused elementwise group with every
// shape, stride and constant baked in as a literal. All kernels requested
// while a graph is planned are compiled together in one NVRTC program (one
// compiler start-up per graph), loaded into the current device's primary
// context and cached for the life of the process by (device, source), so
// identical groups (the same layer pattern repeated, or a second graph of the
// same model) compile once.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <nvrtc.h>

#include <cstdio>
#include <cstdlib>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "kernels.cuh"
#include "runtime.hpp"

namespace tg {

namespace {
std::mutex g_jit_mu;
std::map<std::pair<int, std::string>, void*> g_fn_cache;  // (device, source) -> CUfunction
std::vector<std::shared_ptr<JitFn>> g_pending;

std::string nvrtc_err(nvrtcProgram prog, nvrtcResult r, const char* what) {
  std::string msg = std::string("NVRTC ") + what + ": " + nvrtcGetErrorString(r);
  if (prog) {
    size_t n = 0;
    if (nvrtcGetProgramLogSize(prog, &n) == NVRTC_SUCCESS && n > 1) {
      std::string log(n, '\0');
      nvrtcGetProgramLog(prog, &log[0]);
      msg += "\n" + log.substr(0, 4000);
    }
  }
  return msg;
}
// Driver entry points, resolved through the runtime so that the library
// itself does not depend on libcuda (it loads on machines without a driver,
// where only planning runs).
struct DriverFns {
  PFN_cuModuleLoadData_v2000 load = nullptr;
  PFN_cuModuleGetFunction_v2000 get = nullptr;
  PFN_cuLaunchKernel_v4000 launch = nullptr;
  PFN_cuGetErrorString_v6000 err = nullptr;
};
const DriverFns& drv() {
  static DriverFns d;
  static bool done = false;
  if (!done) {
    auto sym = [](const char* name) -> void* {
      void* p = nullptr;
      cudaDriverEntryPointQueryResult q;
      if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess)
        throw TgError("CudaError", std::string("driver entry point ") + name + " unavailable");
      return p;
    };
    d.load = reinterpret_cast<PFN_cuModuleLoadData_v2000>(sym("cuModuleLoadData"));
    d.get = reinterpret_cast<PFN_cuModuleGetFunction_v2000>(sym("cuModuleGetFunction"));
    d.launch = reinterpret_cast<PFN_cuLaunchKernel_v4000>(sym("cuLaunchKernel"));
    d.err = reinterpret_cast<PFN_cuGetErrorString_v6000>(sym("cuGetErrorString"));
    done = true;
  }
  return d;
}
std::string cu_err(CUresult r) {
  const char* s = nullptr;
  if (drv().err) drv().err(r, &s);
  return s ? s : "CUresult " + std::to_string((int)r);
}
}  // namespace

std::shared_ptr<JitFn> jit_request(const std::string& name, const std::string& src) {
  int dev = 0;
  TG_CUDA(cudaGetDevice(&dev));
  auto f = std::make_shared<JitFn>();
  f->name = name;
  f->src = src;
  f->device = dev;
  std::lock_guard<std::mutex> lk(g_jit_mu);
  auto it = g_fn_cache.find({dev, src});
  if (it != g_fn_cache.end()) f->fn = it->second;
  else g_pending.push_back(f);
  return f;
}

void jit_compile_pending() {
  std::lock_guard<std::mutex> lk(g_jit_mu);
  if (g_pending.empty()) return;
  int dev = 0;
  TG_CUDA(cudaGetDevice(&dev));
  // One translation unit: the shared preamble, then each distinct kernel once.
  std::string tu = jit_preamble();
  std::map<std::string, std::string> by_src;  // source -> kernel name
  for (auto& f : g_pending) {
    if (g_fn_cache.count({dev, f->src})) continue;
    if (by_src.emplace(f->src, f->name).second) tu += f->src;
  }
  if (const char* dump = getenv("TG_JIT_DUMP")) {
    if (FILE* fp = fopen(dump, "a")) { fputs(tu.c_str(), fp); fclose(fp); }
  }
  if (!by_src.empty()) {
    nvrtcProgram prog = nullptr;
    nvrtcResult r = nvrtcCreateProgram(&prog, tu.c_str(), "tg_fused.cu", 0, nullptr, nullptr);
    if (r != NVRTC_SUCCESS) throw TgError("CompileError", nvrtc_err(nullptr, r, "create"));
    const char* opts[] = {"--gpu-architecture=sm_100a", "--std=c++17", "-default-device"};
    r = nvrtcCompileProgram(prog, 3, opts);
    if (r != NVRTC_SUCCESS) {
      std::string m = nvrtc_err(prog, r, "compile");
      nvrtcDestroyProgram(&prog);
      throw TgError("CompileError", m);
    }
    size_t n = 0;
    r = nvrtcGetCUBINSize(prog, &n);
    std::string cubin(n, '\0');
    if (r == NVRTC_SUCCESS) r = nvrtcGetCUBIN(prog, &cubin[0]);
    nvrtcDestroyProgram(&prog);
    if (r != NVRTC_SUCCESS) throw TgError("CompileError", nvrtc_err(nullptr, r, "cubin"));
    CUmodule mod = nullptr;
    CUresult cr = drv().load(&mod, cubin.data());
    if (cr != CUDA_SUCCESS) throw TgError("CudaError", "cuModuleLoadData: " + cu_err(cr));
    for (auto& kv : by_src) {
      CUfunction fn = nullptr;
      cr = drv().get(&fn, mod, kv.second.c_str());
      if (cr != CUDA_SUCCESS) throw TgError("CudaError", "cuModuleGetFunction " + kv.second + ": " + cu_err(cr));
      g_fn_cache[{dev, kv.first}] = fn;
    }
  }
  for (auto& f : g_pending) f->fn = g_fn_cache.at({dev, f->src});
  g_pending.clear();
}

void jit_launch(const JitFn& f, unsigned grid_x, unsigned grid_y, unsigned block, void** args, cudaStream_t s) {
  if (!f.fn) throw TgError("Error", "internal: kernel " + f.name + " was not compiled");
  CUresult r = drv().launch(reinterpret_cast<CUfunction>(f.fn), grid_x, grid_y, 1, block, 1, 1, 0,
                            reinterpret_cast<CUstream>(s), args, nullptr);
  if (r != CUDA_SUCCESS) throw TgError("CudaError", "launch " + f.name + ": " + cu_err(r));
}

// Device helpers every generated kernel may use. Arithmetic goes through the
// round-to-nearest intrinsics so that no multiply-add is contracted and each
// op rounds to f32 exactly as a separate kernel would.
const std::string& jit_preamble() {
  static const std::string s = R"(
typedef unsigned int u32;
typedef long long i64;
__device__ __forceinline__ float f4(const float4& q, int l) { return l == 0 ? q.x : l == 1 ? q.y : l == 2 ? q.z : q.w; }
__device__ __forceinline__ u32 tg_pcg(u32 h) {
  h = h * 747796405u + 2891336453u;
  h = ((h >> ((h >> 28u) + 4u)) ^ h) * 277803737u;
  return (h >> 22u) ^ h;
}
__device__ __forceinline__ float tg_erf(float x) {
  float s = x > 0.f ? 1.f : (x < 0.f ? -1.f : 0.f);
  float ax = fabsf(x);
  float t = 1.0f / (1.0f + 0.3275911f * ax);
  float p = t * (0.254829592f + t * (-0.284496736f + t * (1.421413741f + t * (-1.453152027f + t * 1.061405429f))));
  return s * (1.0f - p * expf(-ax * ax));
}
__device__ __forceinline__ float tg_bits(u32 b) { return __uint_as_float(b); }
)";
  return s;
}

}  // namespace tg
