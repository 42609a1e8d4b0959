// Layout, indexing, conv/pool and optimizer kernels.
//
// Reference counterparts (one WGSL kernel per op there): permute
// (src/codegen.ts:468-493), slice/scatter/concat (:715-819), broadcast_to
// (:822-837), one_hot (:604-624), arange/const fills (:71-104), randn
// (:212-239), max pool + grad (:1095-1185); conv2d lives in kernels_conv.cu,
// Adam (:841-905: three kernels plus three copy-backs per param there; one
// in-place pass over flat arenas here).
#include <algorithm>

#include "kernels.cuh"

namespace tg {

static unsigned grid_for(int64_t work, int threads = 256, int per_sm = 8) {
  int64_t b = (work + threads - 1) / threads;
  int64_t cap = (int64_t)device_sm_count() * per_sm;
  if (b > cap) b = cap;
  if (b < 1) b = 1;
  return (unsigned)b;
}

// ------------------------------------------------------------- strided copy --
__global__ void __launch_bounds__(256) copy_kernel(const __grid_constant__ CopyDesc d, const uint32_t* __restrict__ in,
                                                   uint32_t* __restrict__ out) {
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < d.numel; i += stride) {
    int64_t rem = i, io = 0, oo = 0;
    for (int k = d.rank - 1; k >= 0; --k) {
      int64_t c = rem % d.dims[k];
      rem /= d.dims[k];
      io += c * d.in_strides[k];
      oo += c * d.out_strides[k];
    }
    out[oo] = in[io];
  }
}

void launch_copy(const CopyDesc& d, const void* in, void* out, cudaStream_t s) {
  if (d.numel <= 0) return;
  copy_kernel<<<grid_for(d.numel), 256, 0, s>>>(d, reinterpret_cast<const uint32_t*>(in),
                                                 reinterpret_cast<uint32_t*>(out));
}

// -------------------------------------------------------------- fills etc. --
__global__ void fill_kernel(uint32_t* out, int64_t n, uint32_t bits) {
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) out[i] = bits;
}
void launch_fill(void* out, int64_t n, uint32_t bits, cudaStream_t s) {
  if (n <= 0) return;
  fill_kernel<<<grid_for(n), 256, 0, s>>>(reinterpret_cast<uint32_t*>(out), n, bits);
}

__global__ void scale_kernel(float* x, int64_t n, float sc) {
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) x[i] *= sc;
}
void launch_scale(float* x, int64_t n, float sc, cudaStream_t s) {
  if (n <= 0) return;
  scale_kernel<<<grid_for(n), 256, 0, s>>>(x, n, sc);
}

__global__ void arange_kernel(void* out, int64_t n, int dtype) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  if (dtype == F32) reinterpret_cast<float*>(out)[i] = (float)i;
  else reinterpret_cast<int*>(out)[i] = (int)i;
}
void launch_arange(void* out, int64_t n, int dtype, cudaStream_t s) {
  arange_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(out, n, dtype);
}

__global__ void one_hot_kernel(const int* __restrict__ idx, void* out, int64_t n, int64_t depth, int dtype) {
  int64_t total = n * depth;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    int64_t r = i / depth, d = i % depth;
    bool hot = (int64_t)idx[r] == d;
    if (dtype == F32) reinterpret_cast<float*>(out)[i] = hot ? 1.f : 0.f;
    else reinterpret_cast<int*>(out)[i] = hot ? 1 : 0;
  }
}
void launch_one_hot(const int* idx, void* out, int64_t n_idx, int64_t depth, int dtype, cudaStream_t s) {
  one_hot_kernel<<<grid_for(n_idx * depth), 256, 0, s>>>(idx, out, n_idx, depth, dtype);
}

__device__ __forceinline__ uint32_t pcg_m(uint32_t h) {
  h = h * 747796405u + 2891336453u;
  h = ((h >> ((h >> 28u) + 4u)) ^ h) * 277803737u;
  return (h >> 22u) ^ h;
}

// randn: two chained PCG draws + Box-Muller cos branch (src/codegen.ts:212-239).
__global__ void randn_kernel(float* out, int64_t n, const int* seed, uint32_t salt) {
  uint32_t sd = (uint32_t)(*seed);
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    uint32_t h1 = pcg_m(sd ^ salt ^ (uint32_t)i);
    uint32_t h2 = pcg_m(h1);
    float u1 = fmaxf(1.0e-10f, __uint2float_rn(h1) * 2.3283064365386963e-10f);
    float u2 = __uint2float_rn(h2) * 2.3283064365386963e-10f;
    out[i] = sqrtf(-2.0f * logf(u1)) * cosf(6.283185307179586f * u2);
  }
}
void launch_randn(float* out, int64_t n, const int* seed, uint32_t salt_const, cudaStream_t s) {
  randn_kernel<<<grid_for(n), 256, 0, s>>>(out, n, seed, salt_const);
}

__global__ void gpu_delay_kernel(uint64_t ns) {
  uint64_t t0, t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  do {
    __nanosleep(2000);
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  } while (t - t0 < ns);
}
void launch_gpu_delay(uint64_t ns, cudaStream_t s) { gpu_delay_kernel<<<1, 1, 0, s>>>(ns); }

// ------------------------------------------------------------ embeddings --
// Gather rows: replaces the reference's oneHot(idx) @ table contraction
// (src/ops.ts:626-635) with a row copy; float4 when D % 4 == 0.
__global__ void __launch_bounds__(256) gather_rows_kernel(const int* __restrict__ idx, const float* __restrict__ table,
                                                          float* __restrict__ out, int64_t rows, int64_t V,
                                                          int64_t D) {
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  if ((D & 3) == 0) {
    int64_t D4 = D >> 2;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < rows * D4; i += stride) {
      int64_t r = i / D4, c = i % D4;
      int64_t v = idx[r];
      float4 val = (v >= 0 && v < V) ? __ldg(reinterpret_cast<const float4*>(table + v * D) + c)
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
      reinterpret_cast<float4*>(out)[i] = val;
    }
  } else {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < rows * D; i += stride) {
      int64_t r = i / D, c = i % D;
      int64_t v = idx[r];
      out[i] = (v >= 0 && v < V) ? table[v * D + c] : 0.f;
    }
  }
}
// Rows of D % 4 == 0 and D <= 1024: a warp per row, lanes over the row's
// float4s (no 64-bit division per element), 8 rows per block.
__global__ void __launch_bounds__(256) gather_rows4_kernel(const int* __restrict__ idx, const float* __restrict__ table,
                                                           float* __restrict__ out, int64_t rows, int64_t V, int D4) {
  const int lane = threadIdx.x & 31;
  for (int64_t r = ((int64_t)blockIdx.x * 256 + threadIdx.x) >> 5; r < rows; r += ((int64_t)gridDim.x * 256) >> 5) {
    const int64_t v = __ldg(idx + r);
    const bool ok = v >= 0 && v < V;
    const float4* src = reinterpret_cast<const float4*>(table + (ok ? v : 0) * D4 * 4);
    float4* dst = reinterpret_cast<float4*>(out + r * D4 * 4);
    for (int c = lane; c < D4; c += 32) dst[c] = ok ? __ldg(src + c) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
}
void launch_gather_rows(const int* idx, const float* table, float* out, int64_t rows, int64_t V, int64_t D,
                        cudaStream_t s) {
  if ((D & 3) == 0 && D <= 4096 && ((uintptr_t)table & 15) == 0 && ((uintptr_t)out & 15) == 0) {
    gather_rows4_kernel<<<grid_for(rows * 32), 256, 0, s>>>(idx, table, out, rows, V, (int)(D >> 2));
    return;
  }
  gather_rows_kernel<<<grid_for(rows * D / ((D & 3) == 0 ? 4 : 1)), 256, 0, s>>>(idx, table, out, rows, V, D);
}

// Deterministic embedding backward (replaces the reference's dB matmul of
// the one-hot, src/grad.ts:407-427): a stable counting sort groups row ids by
// vocabulary id, then each vocabulary row sums its rows of dy in ascending row
// order. No float atomics, so results are bit-reproducible run to run (the
// reference avoided atomics for the same reason, src/nn.ts:79-81).
//
// Scratch (ints): perm[rows] | cnt[nchunk * V] | start[V + 1] | (256 B aligned)
// segment partial sums (floats) [segments][V][D] when the float4 path splits
// each bucket into segments.
static const int64_t EMB_CHUNK = 1024;
static int64_t emb_chunks(int64_t rows) { return (rows + EMB_CHUNK - 1) / EMB_CHUNK; }
// Segments per bucket for the float4 sum: enough warps to keep the SMs busy
// when the vocabulary is small (C4: 65 rows of 384 columns, about 250 rows per
// bucket), one when it is large.
static int64_t emb_segments(int64_t rows, int64_t V, int64_t D) {
  if (D % 4 != 0 || V <= 0) return 1;
  const int64_t units = V * ((D / 4 + 31) / 32);
  const int64_t want = (int64_t)device_sm_count() * 32;
  int64_t s = want / std::max<int64_t>(units, 1);
  s = std::min<int64_t>(s, std::max<int64_t>(1, rows / std::max<int64_t>(V, 1) / 16));
  return std::max<int64_t>(1, std::min<int64_t>(s, 16));
}
static int64_t emb_head_ints(int64_t rows, int64_t V) {
  return (rows + emb_chunks(rows) * V + V + 1 + 63) / 64 * 64;
}
size_t embedding_grad_scratch_ints(int64_t rows, int64_t V, int64_t D) {
  const int64_t s = emb_segments(rows, V, D);
  return (size_t)(emb_head_ints(rows, V) + (s > 1 ? s * V * D : 0));
}

__global__ void emb_hist_kernel(const int* __restrict__ idx, int* __restrict__ cnt, int64_t rows, int64_t V) {
  int64_t c = blockIdx.x;
  int64_t r0 = c * EMB_CHUNK, r1 = r0 + EMB_CHUNK < rows ? r0 + EMB_CHUNK : rows;
  for (int64_t r = r0 + threadIdx.x; r < r1; r += blockDim.x) {
    int64_t v = idx[r];
    if (v >= 0 && v < V) atomicAdd(&cnt[c * V + v], 1);
  }
}
// per bucket: chunk counts -> exclusive offsets inside the bucket; total -> start[v]
__global__ void emb_bucket_kernel(int* __restrict__ cnt, int* __restrict__ start, int64_t nchunk, int64_t V) {
  int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (v >= V) return;
  int run = 0;
  for (int64_t c = 0; c < nchunk; ++c) {
    int k = cnt[c * V + v];
    cnt[c * V + v] = run;
    run += k;
  }
  start[v] = run;
}
// exclusive scan of start[0..V) in one block; start[V] = total
__global__ void emb_scan_kernel(int* __restrict__ start, int64_t V) {
  __shared__ int wsum[32];
  __shared__ int carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  for (int64_t base = 0; base < V; base += blockDim.x) {
    int64_t i = base + threadIdx.x;
    int c = i < V ? start[i] : 0;
    int x = c;
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) wsum[wid] = x;
    __syncthreads();
    if (wid == 0) {
      int w = lane < (int)(blockDim.x >> 5) ? wsum[lane] : 0;
      for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      wsum[lane] = w;
    }
    __syncthreads();
    int incl = x + (wid > 0 ? wsum[wid - 1] : 0);
    int cbase = carry;
    __syncthreads();
    if (i < V) start[i] = cbase + incl - c;
    if (threadIdx.x == blockDim.x - 1) carry = cbase + incl;
    __syncthreads();
  }
  if (threadIdx.x == 0) start[V] = carry;
}
// one warp per chunk places its rows in row order (stable)
__global__ void emb_place_kernel(const int* __restrict__ idx, int* __restrict__ cnt, const int* __restrict__ start,
                                 int* __restrict__ perm, int64_t rows, int64_t V) {
  int64_t c = blockIdx.x;
  int lane = threadIdx.x;
  int64_t r0 = c * EMB_CHUNK, r1 = r0 + EMB_CHUNK < rows ? r0 + EMB_CHUNK : rows;
  int* cur = cnt + c * V;
  for (int64_t base = r0; base < r1; base += 32) {
    int64_t r = base + lane;
    int v = r < r1 ? idx[r] : -1;
    bool ok = r < r1 && v >= 0 && v < V;
    unsigned same = __match_any_sync(0xffffffffu, ok ? v : -1);
    int rank = __popc(same & ((1u << lane) - 1u));
    int pos = ok ? start[v] + cur[v] + rank : 0;
    __syncwarp();
    bool last = (same >> lane) == 1u;
    if (ok && last) cur[v] += rank + 1;
    __syncwarp();
    if (ok) perm[pos] = (int)r;
  }
}
__global__ void __launch_bounds__(256) emb_sum_kernel(const int* __restrict__ start, const int* __restrict__ perm,
                                                      const float* __restrict__ dy, float* __restrict__ dtable,
                                                      int64_t V, int64_t D) {
  for (int64_t v = blockIdx.x; v < V; v += gridDim.x) {
    int s0 = start[v], s1 = start[v + 1];
    for (int64_t c = threadIdx.x; c < D; c += blockDim.x) {
      float acc = 0.f;
      for (int k = s0; k < s1; ++k) acc += dy[(int64_t)perm[k] * D + c];
      dtable[v * D + c] = acc;
    }
  }
}
// D % 4 == 0: one warp per (vocabulary row, 128 columns, segment of the
// bucket), four columns per lane, the segment's rows in ascending order,
// eight rows' loads issued before their adds. With several segments each
// writes a partial row and emb_fold4_kernel adds them in segment order: a
// fixed order, so the result is deterministic.
__global__ void __launch_bounds__(256) emb_sum4_kernel(const int* __restrict__ start, const int* __restrict__ perm,
                                                       const float* __restrict__ dy, float* __restrict__ dtable,
                                                       int64_t V, int D4, int nseg, float* __restrict__ part) {
  const int lane = threadIdx.x & 31;
  const int cb = (D4 + 31) / 32;
  const int64_t units = V * cb * nseg;
  for (int64_t u = ((int64_t)blockIdx.x * 256 + threadIdx.x) >> 5; u < units; u += ((int64_t)gridDim.x * 256) >> 5) {
    const int sg = (int)(u % nseg);
    const int64_t vc = u / nseg;
    const int64_t v = vc / cb;
    const int c = (int)(vc % cb) * 32 + lane;
    const int b0 = __ldg(start + v), b1 = __ldg(start + v + 1);
    const int64_t len = b1 - b0;
    const int s0 = b0 + (int)(len * sg / nseg), s1 = b0 + (int)(len * (sg + 1) / nseg);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (c < D4) {
      const float4* src = reinterpret_cast<const float4*>(dy) + c;
      int k = s0;
      for (; k + 8 <= s1; k += 8) {
        float4 x[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) x[q] = __ldg(src + (int64_t)__ldg(perm + k + q) * D4);
#pragma unroll
        for (int q = 0; q < 8; ++q) { acc.x += x[q].x; acc.y += x[q].y; acc.z += x[q].z; acc.w += x[q].w; }
      }
      for (; k < s1; ++k) {
        const float4 x = __ldg(src + (int64_t)__ldg(perm + k) * D4);
        acc.x += x.x; acc.y += x.y; acc.z += x.z; acc.w += x.w;
      }
      float* dst = nseg > 1 ? part + ((int64_t)sg * V + v) * D4 * 4 : dtable + v * D4 * 4;
      reinterpret_cast<float4*>(dst)[c] = acc;
    }
  }
}

__global__ void __launch_bounds__(256) emb_fold4_kernel(const float* __restrict__ part, float* __restrict__ dtable,
                                                        int64_t n4, int nseg) {
  for (int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x; i < n4; i += (int64_t)gridDim.x * 256) {
    float4 a = __ldg(reinterpret_cast<const float4*>(part) + i);
    for (int sg = 1; sg < nseg; ++sg) {
      const float4 b = __ldg(reinterpret_cast<const float4*>(part) + sg * n4 + i);
      a.x += b.x; a.y += b.y; a.z += b.z; a.w += b.w;
    }
    reinterpret_cast<float4*>(dtable)[i] = a;
  }
}

void launch_embedding_grad(const int* idx, const float* dy, float* dtable, int64_t rows, int64_t V, int64_t D,
                           int* scratch, cudaStream_t s) {
  int64_t nchunk = emb_chunks(rows);
  int* perm = scratch;
  int* cnt = scratch + rows;
  int* start = cnt + nchunk * V;
  cudaMemsetAsync(cnt, 0, sizeof(int) * (size_t)(nchunk * V), s);
  if (nchunk > 0) emb_hist_kernel<<<(unsigned)nchunk, 256, 0, s>>>(idx, cnt, rows, V);
  emb_bucket_kernel<<<(unsigned)((V + 255) / 256), 256, 0, s>>>(cnt, start, nchunk, V);
  emb_scan_kernel<<<1, 1024, 0, s>>>(start, V);
  if (nchunk > 0) emb_place_kernel<<<(unsigned)nchunk, 32, 0, s>>>(idx, cnt, start, perm, rows, V);
  if ((D & 3) == 0 && ((uintptr_t)dy & 15) == 0 && ((uintptr_t)dtable & 15) == 0) {
    const int nseg = (int)emb_segments(rows, V, D);
    float* part = reinterpret_cast<float*>(scratch + emb_head_ints(rows, V));
    const int64_t units = V * ((D / 4 + 31) / 32) * nseg;
    emb_sum4_kernel<<<grid_for(units * 32), 256, 0, s>>>(start, perm, dy, dtable, V, (int)(D / 4), nseg, part);
    if (nseg > 1) emb_fold4_kernel<<<grid_for(V * D / 4), 256, 0, s>>>(part, dtable, V * D / 4, nseg);
    return;
  }
  int64_t cap = (int64_t)device_sm_count() * 16;
  int64_t blocks = V < cap ? V : cap;
  emb_sum_kernel<<<(unsigned)(blocks < 1 ? 1 : blocks), 256, 0, s>>>(start, perm, dy, dtable, V, D);
}

__global__ void pick_kernel(const float* __restrict__ x, const int* __restrict__ t, float* __restrict__ out,
                            int64_t rows, int64_t V) {
  int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  int64_t k = t[r];
  out[r] = (k >= 0 && k < V) ? x[r * V + k] : 0.f;
}
void launch_pick(const float* x, const int* t, float* out, int64_t rows, int64_t V, cudaStream_t s) {
  pick_kernel<<<(unsigned)((rows + 255) / 256), 256, 0, s>>>(x, t, out, rows, V);
}

// out[r] = g[r] where 0 <= t[r] < V, else 0: the row sum of g[r] * oneHot(t)[r].
__global__ void row_hit_kernel(const float* __restrict__ g, const int* __restrict__ t, float* __restrict__ out,
                               int64_t rows, int64_t V) {
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  const int k = t[r];
  out[r] = (k >= 0 && k < V) ? g[r] : 0.f;
}
void launch_row_hit(const float* g, const int* t, float* out, int64_t rows, int64_t V, cudaStream_t s) {
  row_hit_kernel<<<(unsigned)((rows + 255) / 256), 256, 0, s>>>(g, t, out, rows, V);
}

// ------------------------------------------------------------- conv / pool --
// Max pool with the reference's scan order and strict '>' from -3.4e38, so
// the first maximum wins (test/_eval.ts:716-738).
__global__ void maxpool_kernel(const __grid_constant__ ConvDesc c, const float* __restrict__ x, float* __restrict__ y) {
  int64_t total = (int64_t)c.B * c.Cin * c.Hout * c.Wout;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    int wo = i % c.Wout;
    int ho = (i / c.Wout) % c.Hout;
    int64_t bc = i / ((int64_t)c.Wout * c.Hout);
    const float* xb = x + bc * c.H * c.W;
    float m = -3.4e38f;
    for (int kh = 0; kh < c.kH; ++kh) {
      int hi = ho * c.sH + kh - c.pH;
      if (hi < 0 || hi >= c.H) continue;
      for (int kw = 0; kw < c.kW; ++kw) {
        int wi = wo * c.sW + kw - c.pW;
        if (wi < 0 || wi >= c.W) continue;
        float v = xb[hi * c.W + wi];
        if (v > m) m = v;
      }
    }
    y[i] = m;
  }
}
void launch_maxpool(const ConvDesc& c, const float* x, float* y, cudaStream_t s) {
  maxpool_kernel<<<grid_for((int64_t)c.B * c.Cin * c.Hout * c.Wout), 256, 0, s>>>(c, x, y);
}

// Gather form (one thread per input element, no atomics), recomputing each
// covering window's argmax exactly as the forward scans it
// (test/_eval.ts:739-779).
__global__ void maxpool_grad_kernel(const __grid_constant__ ConvDesc c, const float* __restrict__ x,
                                    const float* __restrict__ dy, float* __restrict__ dx) {
  int64_t total = (int64_t)c.B * c.Cin * c.H * c.W;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    int wi = i % c.W;
    int hi = (i / c.W) % c.H;
    int64_t bc = i / ((int64_t)c.W * c.H);
    const float* xb = x + bc * c.H * c.W;
    const float* db = dy + bc * c.Hout * c.Wout;
    float s = 0.f;
    for (int kh = 0; kh < c.kH; ++kh) {
      int nh = hi + c.pH - kh;
      if (nh < 0 || nh % c.sH) continue;
      int ho = nh / c.sH;
      if (ho >= c.Hout) continue;
      for (int kw = 0; kw < c.kW; ++kw) {
        int nw = wi + c.pW - kw;
        if (nw < 0 || nw % c.sW) continue;
        int wo = nw / c.sW;
        if (wo >= c.Wout) continue;
        float m = -3.4e38f;
        int ah = -1, aw = -1;
        for (int a = 0; a < c.kH; ++a) {
          int hh = ho * c.sH + a - c.pH;
          if (hh < 0 || hh >= c.H) continue;
          for (int b2 = 0; b2 < c.kW; ++b2) {
            int ww = wo * c.sW + b2 - c.pW;
            if (ww < 0 || ww >= c.W) continue;
            float v = xb[hh * c.W + ww];
            if (v > m) { m = v; ah = hh; aw = ww; }
          }
        }
        if (ah == hi && aw == wi) s += db[ho * c.Wout + wo];
      }
    }
    dx[i] = s;
  }
}
// Windows that do not overlap (stride >= window on both axes): each input
// element lies in at most one window, found directly; 32-bit indexing. The
// window's first maximum is recomputed with the forward's scan order.
__global__ void __launch_bounds__(256) maxpool_grad_disjoint_kernel(const __grid_constant__ ConvDesc c,
                                                                    const float* __restrict__ x,
                                                                    const float* __restrict__ dy,
                                                                    float* __restrict__ dx) {
  const int total = c.B * c.Cin * c.H * c.W;
  const int hw = c.H * c.W;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int bc = i / hw, r = i - bc * hw;
    const int hi = r / c.W, wi = r - hi * c.W;
    const int nh = hi + c.pH, nw = wi + c.pW;
    const int ho = nh / c.sH, wo = nw / c.sW;
    float v = 0.f;
    if (nh - ho * c.sH < c.kH && nw - wo * c.sW < c.kW && ho < c.Hout && wo < c.Wout) {
      const float* xb = x + (int64_t)bc * hw;
      float m = -3.4e38f;
      int ah = -1, aw = -1;
      for (int a = 0; a < c.kH; ++a) {
        const int hh = ho * c.sH + a - c.pH;
        if (hh < 0 || hh >= c.H) continue;
        for (int b2 = 0; b2 < c.kW; ++b2) {
          const int ww = wo * c.sW + b2 - c.pW;
          if (ww < 0 || ww >= c.W) continue;
          const float xv = xb[hh * c.W + ww];
          if (xv > m) { m = xv; ah = hh; aw = ww; }
        }
      }
      if (ah == hi && aw == wi) v = dy[(int64_t)bc * c.Hout * c.Wout + ho * c.Wout + wo];
    }
    dx[i] = v;
  }
}

// 2x2 windows, stride 2, no padding, tiling the input exactly: one thread
// per window reads its four inputs (two float2 loads), picks the first
// maximum in the forward's scan order (from -3.4e38 with strict '>', so a
// window with no element above that routes no gradient) and writes dy there
// and 0 elsewhere.
__global__ void __launch_bounds__(256) maxpool2_grad_kernel(int planes, int Hout, int Wout,
                                                            const float* __restrict__ x,
                                                            const float* __restrict__ dy, float* __restrict__ dx) {
  const int total = planes * Hout * Wout, W = 2 * Wout;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int pl = i / (Hout * Wout), r = i - pl * (Hout * Wout);
    const int ho = r / Wout, wo = r - ho * Wout;
    const int64_t top = (int64_t)pl * (4 * Hout * Wout) + (2 * ho) * W + 2 * wo;
    const float2 a = *reinterpret_cast<const float2*>(x + top);
    const float2 b = *reinterpret_cast<const float2*>(x + top + W);
    float m = -3.4e38f;
    int at = -1;
    if (a.x > m) { m = a.x; at = 0; }
    if (a.y > m) { m = a.y; at = 1; }
    if (b.x > m) { m = b.x; at = 2; }
    if (b.y > m) { m = b.y; at = 3; }
    const float g = dy[i];
    *reinterpret_cast<float2*>(dx + top) = make_float2(at == 0 ? g : 0.f, at == 1 ? g : 0.f);
    *reinterpret_cast<float2*>(dx + top + W) = make_float2(at == 2 ? g : 0.f, at == 3 ? g : 0.f);
  }
}

void launch_maxpool_grad(const ConvDesc& c, const float* x, const float* dy, float* dx, cudaStream_t s) {
  const int64_t total = (int64_t)c.B * c.Cin * c.H * c.W;
  if (c.kH == 2 && c.kW == 2 && c.sH == 2 && c.sW == 2 && c.pH == 0 && c.pW == 0 && c.H == 2 * c.Hout &&
      c.W == 2 * c.Wout && total < INT32_MAX && !(reinterpret_cast<uintptr_t>(x) & 7) &&
      !(reinterpret_cast<uintptr_t>(dx) & 7))
    maxpool2_grad_kernel<<<grid_for(total / 4, 256, 16), 256, 0, s>>>(c.B * c.Cin, c.Hout, c.Wout, x, dy, dx);
  else if (c.sH >= c.kH && c.sW >= c.kW && total < INT32_MAX)
    maxpool_grad_disjoint_kernel<<<grid_for(total, 256, 16), 256, 0, s>>>(c, x, dy, dx);
  else
    maxpool_grad_kernel<<<grid_for(total), 256, 0, s>>>(c, x, dy, dx);
}

// dst[r * ld_dst + c] = src[r * ld_src + c] for r < rows, c < cols: an
// operand copied to 16-byte row strides so TMA can describe it.
__global__ void __launch_bounds__(256) pad_rows_kernel(const float* __restrict__ src, int64_t ld_src,
                                                       float* __restrict__ dst, int64_t ld_dst, int64_t rows,
                                                       int64_t cols) {
  const int64_t total = rows * cols;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cols, c = i - r * cols;
    dst[r * ld_dst + c] = src[r * ld_src + c];
  }
}
void launch_pad_rows(const float* src, int64_t ld_src, float* dst, int64_t ld_dst, int64_t rows, int64_t cols,
                     cudaStream_t s) {
  if (rows <= 0 || cols <= 0) return;
  pad_rows_kernel<<<grid_for(rows * cols), 256, 0, s>>>(src, ld_src, dst, ld_dst, rows, cols);
}

// ------------------------------------------------------------ optimizers --
// One in-place pass over the flat param/grad/moment arenas: reads p, g, m, v
// once and writes p, m, v once (28 bytes per parameter), float4-wide. Arena
// lengths are padded to a multiple of 4 floats with zeros.
__global__ void __launch_bounds__(256) adam_flat_kernel(const __grid_constant__ AdamFlatDesc d) {
  float lrt = *d.lrt;
  float shrink = d.shrink_dev ? *d.shrink_dev : d.shrink_lit;
  int64_t n4 = d.n >> 2;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < n4; q += stride) {
    float4 p = reinterpret_cast<float4*>(d.p)[q];
    float4 g = reinterpret_cast<const float4*>(d.g)[q];
    float4 m = reinterpret_cast<float4*>(d.m)[q];
    float4 v = reinterpret_cast<float4*>(d.v)[q];
    float* pp = &p.x; float* gg = &g.x; float* mm = &m.x; float* vv = &v.x;
#pragma unroll
    for (int l = 0; l < 4; ++l) {
      int64_t e = (q << 2) + l;
      float gl = gg[l] * d.grad_scale;
      float mn = d.beta1 * mm[l] + d.one_minus_beta1 * gl;
      float vn = d.beta2 * vv[l] + d.one_minus_beta2 * gl * gl;
      float sh = e < d.n_decay ? shrink : 1.0f;
      pp[l] = sh * pp[l] - __fdiv_rn(lrt * mn, __fsqrt_rn(vn) + d.eps);
      mm[l] = mn;
      vv[l] = vn;
    }
    reinterpret_cast<float4*>(d.p)[q] = p;
    reinterpret_cast<float4*>(d.m)[q] = m;
    reinterpret_cast<float4*>(d.v)[q] = v;
  }
}
void launch_adam_flat(const AdamFlatDesc& d, cudaStream_t s) {
  adam_flat_kernel<<<grid_for(d.n / 4), 256, 0, s>>>(d);
}

__global__ void __launch_bounds__(256) sgd_flat_kernel(const __grid_constant__ SgdFlatDesc d) {
  float lr = *d.lr;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < d.n; e += stride) {
    float p = d.p[e];
    float g = d.g[e] * d.grad_scale;
    if (e < d.n_decay) g = g + p * d.wd;
    float upd = g;
    if (d.v) {
      float vn = d.v[e] * d.momentum + g;
      d.v[e] = vn;
      upd = d.nesterov ? g + vn * d.momentum : vn;
    }
    d.p[e] = p - lr * upd;
  }
}
void launch_sgd_flat(const SgdFlatDesc& d, cudaStream_t s) {
  sgd_flat_kernel<<<grid_for(d.n), 256, 0, s>>>(d);
}

}  // namespace tg
