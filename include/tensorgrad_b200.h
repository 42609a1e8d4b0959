/* tensorgrad_b200 — C ABI of the B200 execution backend (libtgcuda.so).
 *
 * This is the boundary the reference's worker would bind in place of its
 * WebGPU runtime. Each entry point replaces one reference interface:
 *
 *   tg_ctx_create / tg_ctx_destroy   ensureDevice + the worker's device
 *                                    ownership (src/worker.ts:58-82)
 *   tg_nccl_unique_id                (new: data-parallel rendezvous token)
 *   tg_graph_create                  createRuntime(plan, kernels, ...)
 *                                    (src/runtime.ts:157-162) fed the traced
 *                                    graph instead of WGSL kernels; the
 *                                    worker's handleCreateRuntime /
 *                                    handleCompileForward (src/worker.ts:86-170)
 *   tg_graph_info                    CompiledRuntime.params/outputShape
 *                                    (src/runtime.ts:123-137)
 *   tg_upload_params                 uploadParams (src/runtime.ts:403-429)
 *   tg_download_params               downloadParams (src/runtime.ts:431-449)
 *   tg_step                          handleStep -> runtime.step
 *                                    (src/worker.ts:216-240, src/runtime.ts:388-393)
 *   tg_run                           handleRun -> runtime.run
 *                                    (src/worker.ts:242-260, src/runtime.ts:395-400)
 *   tg_set_inputs / tg_launch_step /
 *   tg_read_loss / tg_stream         the three phases of dispatchUnsynchronized
 *                                    (src/runtime.ts:314-386), split so a caller
 *                                    can keep inputs resident and pipeline steps
 *   tg_reset_optimizer               resetOptimizerState (src/runtime.ts:461-465,
 *                                    src/worker.ts:295-302)
 *   tg_set_lr                        handleSetLR (src/worker.ts:304-319)
 *   tg_destroy_graph                 destroy + cascade (src/worker.ts:321-334)
 *   tg_read_grad / tg_read_tensor    (new: inspection for parity tests)
 *   tg_launch_list / tg_profile_step (new: per-kernel launch list and timing;
 *                                    the reference labels its compute passes
 *                                    for browser profilers, src/runtime.ts:340)
 *   tg_last_error_name/_message      the worker's serialized {name, message}
 *                                    errors (src/worker-protocol.ts:118-177)
 *
 * All functions return 0 on success and a nonzero status otherwise; the
 * thread-local error name/message describe the failure. Host pointers stay
 * owned by the caller. A context is used from one thread at a time.
 */
#ifndef TENSORGRAD_B200_H
#define TENSORGRAD_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct tg_ctx tg_ctx;

enum {
  TG_OK = 0,
  TG_ERR = 1,       /* "Error" */
  TG_ABORTED = 2,   /* "AbortError": graph destroyed or replaced mid-call */
  TG_CUDA_ERR = 3,  /* "CudaError" */
  TG_NCCL_ERR = 4,  /* "NcclError" */
};

int tg_nccl_unique_id(uint8_t out[128]);
int tg_ctx_create(int device, int rank, int world, const uint8_t* nccl_id, tg_ctx** out);
int tg_ctx_destroy(tg_ctx* ctx);

/* program_json: {"graph": WireIR graph, "params", "inputs", "states",
 * "paramGrads", "writebacks", "loss", "optimizer", "usesPrng", "optStart"}.
 * parent_graph_id = -1 owns its params; otherwise params are shared with
 * that graph (a forward sibling). */
int tg_graph_create(tg_ctx* ctx, int graph_id, int parent_graph_id, const char* program_json, size_t len);
/* Writes a JSON description into buf (params, launch count, device bytes). */
int tg_graph_info(tg_ctx* ctx, int graph_id, char* buf, size_t cap, size_t* needed);
int tg_upload_params(tg_ctx* ctx, int graph_id, int n, const char* const* names, const float* const* data,
                     const size_t* numel);
int tg_download_params(tg_ctx* ctx, int graph_id, int n, const char* const* names, float* const* out,
                       const size_t* numel);
/* One synchronous training step from host inputs: H2D, kernels, loss D2H.
 * Every declared input must be given (the runtime-written PRNG seed and
 * optimizer scalars excepted), each with its exact byte size. */
int tg_step(tg_ctx* ctx, int graph_id, int n, const char* const* names, const void* const* data,
            const size_t* bytes, float* loss_out, void* const* capture_out);
/* One forward run: output (and captures) copied into caller buffers. Same
 * input rules as tg_step. */
int tg_run(tg_ctx* ctx, int graph_id, int n, const char* const* names, const void* const* data,
           const size_t* bytes, void* output_out, void* const* capture_out);
/* Split step: copy inputs (device_src != 0: data are device pointers),
 * enqueue a step without waiting, read the last loss (synchronizes). */
int tg_set_inputs(tg_ctx* ctx, int graph_id, int n, const char* const* names, const void* const* data,
                  const size_t* bytes, int device_src);
int tg_launch_step(tg_ctx* ctx, int graph_id);
int tg_read_loss(tg_ctx* ctx, int graph_id, float* loss_out);
int tg_stream(tg_ctx* ctx, void** stream_out);
int tg_reset_optimizer(tg_ctx* ctx, int graph_id);
/* Optimizer state by state name (adam_m_<param>, adam_v_<param>,
 * sgd_v_<param>), strict like the param calls; with tg_get_counters /
 * tg_set_counters (optimizer steps taken, PRNG seed counter) this is the
 * training checkpoint. New: the reference exports no optimizer state and its
 * reset re-initialises it (src/compile.ts:641-657; src/runtime.ts:461-465). */
int tg_upload_states(tg_ctx* ctx, int graph_id, int n, const char* const* names, const float* const* data,
                     const size_t* numel);
int tg_download_states(tg_ctx* ctx, int graph_id, int n, const char* const* names, float* const* out,
                       const size_t* numel);
int tg_get_counters(tg_ctx* ctx, int graph_id, int64_t* step, int64_t* prng);
int tg_set_counters(tg_ctx* ctx, int graph_id, int64_t step, int64_t prng);
int tg_set_lr(tg_ctx* ctx, int graph_id, const char* lr_json, size_t len);
int tg_destroy_graph(tg_ctx* ctx, int graph_id);
int tg_read_grad(tg_ctx* ctx, int graph_id, const char* name, float* out);
int tg_read_tensor(tg_ctx* ctx, int graph_id, int tensor_id, void* out);
/* Newline-separated kind of every kernel launch in one step. */
int tg_launch_list(tg_ctx* ctx, int graph_id, char* buf, size_t cap, size_t* needed);

/* Plans a program without a GPU and writes JSON {"info", "launches",
 * "kernelSources", "kernelPreamble"}: the graph info, the label of every
 * launch one step would make, the CUDA source of every fused elementwise
 * kernel and the helper preamble they are compiled with. No device
 * memory is allocated and nothing is compiled or run. No counterpart in the
 * reference (its codegen.ts plan is only visible through the WGSL it emits);
 * used to test planner decisions on machines without a GPU. */
int tg_plan_dry(const char* program_json, size_t len, int world, char* buf, size_t cap, size_t* needed);

/* Runs one step launch by launch with CUDA events around each launch and
 * writes per-launch milliseconds (in tg_launch_list order). */
int tg_profile_step(tg_ctx* ctx, int graph_id, float* ms_out, int cap, int* n_out);

/* Algorithmic bytes of every launch of one step, in tg_launch_list order:
 * each distinct tensor the launch reads counted once at its own size, plus
 * every tensor it writes; 0 for launches not accounted in bytes (GEMMs,
 * convolutions, collectives). Divided by tg_profile_step's times it gives
 * each memory-bound kernel's achieved bandwidth. (new: measurement) */
int tg_launch_bytes(tg_ctx* ctx, int graph_id, double* out, int cap, int* n_out);

/* Error code recorded by a tcgen05 kernel whose bounded barrier wait ran out
 * (0 = none): the GEMM's code in the low byte, the attention forward's
 * shifted left by 8; reset != 0 clears both. (new: kernel health check for
 * tests) */
int tg_debug_gemm_error(int reset);
/* Progress markers of the first GEMM tile (8 ints) for pipeline diagnosis. */
int tg_debug_gemm_dbg(int* out8);
/* Pipeline timeline (SM clock cycles) of the first CTA of the last tcgen05
 * GEMM launched with TG_GEMM_TRACE=1 in the environment: 6 rows of 64
 * (TMA issued, stage landed, split done, MMAs issued per K-stage; chunk
 * drained; start / epilogue start / epilogue end). Returns the number of
 * values written (384) or -1. Debugging aid with no reference counterpart. */
int tg_debug_gemm_trace(long long* out, int cap);

/* Column sums of a row-major [outer, inner] f32 matrix already on the device
 * (out[j] = sum_i x[i*inner + j]), enqueued on `stream` (a cudaStream_t; NULL
 * for the legacy default stream), without allocating anything. It has no
 * counterpart in the reference: it serves callers that may not allocate
 * device memory, such as a host whose pool or caching allocator owns all of
 * the GPU's memory, or a latency-critical loop that must not call cudaMalloc
 * because it can synchronize the device. The deterministic two-pass kernel's
 * partial sums live in a fixed 256 Ki-float (1 MiB) device array that every
 * GPU loading the library holds until exit; shapes that need more partial
 * sums than that are rejected with an error. The first call on each device
 * looks up the array's address and should come before any stream capture.
 * All calls share the array: calls that overlap on the GPU race. */
int tg_colsum_noalloc(const float* x, float* out, int64_t outer, int64_t inner, void* stream);

const char* tg_last_error_name(void);
const char* tg_last_error_message(void);

#ifdef __cplusplus
}
#endif

#endif /* TENSORGRAD_B200_H */
