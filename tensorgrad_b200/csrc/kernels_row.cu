// Row kernels: last-axis reductions and softmaxes (reference: src/codegen.ts
// :333-445 sum/mean/argmax/categorical, :627-689 logSoftmax/softmaxCausal,
// :907-913 + :1383-1477 sum_to_shape), re-designed for B200.
//
// One warp per row when the row fits a warp comfortably (D <= 2048), one
// 256-thread block per row otherwise; warp-shuffle trees, f32 accumulation.
// A few very long rows (the loss mean, global-norm sums) split across CTAs
// into a scratch buffer and finish in a second pass, so the reduction never
// runs on a single SM. Column sums (bias / LayerNorm-gain gradients) are a
// deterministic two-pass reduction: chunked partial sums, then a fold.
#include "kernels.cuh"

namespace tg {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
// (value, index) max with ties broken toward the lower index.
__device__ __forceinline__ void warp_argmax(float& v, int& idx) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, v, o);
    int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > v || (ov == v && oi < idx)) { v = ov; idx = oi; }
  }
}
// Online-softmax merge of (max, sum) pairs across a warp.
__device__ __forceinline__ void warp_online(float& m, float& s) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float om = __shfl_xor_sync(0xffffffffu, m, o);
    float os = __shfl_xor_sync(0xffffffffu, s, o);
    float nm = fmaxf(m, om);
    float a = (m == -INFINITY) ? 0.f : s * expf(m - nm);
    float b = (om == -INFINITY) ? 0.f : os * expf(om - nm);
    m = nm;
    s = a + b;
  }
}

__device__ __forceinline__ uint32_t pcg_r(uint32_t h) {
  h = h * 747796405u + 2891336453u;
  h = ((h >> ((h >> 28u) + 4u)) ^ h) * 277803737u;
  return (h >> 22u) ^ h;
}

// Gumbel-perturbed logit for categorical sampling (src/codegen.ts:409-445).
__device__ __forceinline__ float gumbel_val(float v, uint32_t sd, uint32_t salt, int64_t flat) {
  uint32_t h = pcg_r(sd ^ salt ^ (uint32_t)flat);
  float u = fmaxf(1.0e-10f, __uint2float_rn(h) * 2.3283064365386963e-10f);
  return v + (-logf(-logf(u)));
}

template <int KIND>
__global__ void __launch_bounds__(256) row_warp_kernel(const float* __restrict__ x, void* __restrict__ out,
                                                       int64_t rows, int64_t D, const int* seed, uint32_t salt) {
  int lane = threadIdx.x & 31;
  int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t r = warp; r < rows; r += nwarps) {
    const float* xr = x + r * D;
    if (KIND == ROW_SUM || KIND == ROW_MEAN) {
      float s = 0.f;
      for (int64_t j = lane; j < D; j += 32) s += xr[j];
      s = warp_sum(s);
      if (lane == 0) reinterpret_cast<float*>(out)[r] = KIND == ROW_MEAN ? __fdiv_rn(s, (float)D) : s;
    } else if (KIND == ROW_ARGMAX || KIND == ROW_CATEGORICAL) {
      float best = -INFINITY;
      int bi = 0x7fffffff;
      uint32_t sd = (KIND == ROW_CATEGORICAL && seed) ? (uint32_t)(*seed) : 0u;
      for (int64_t j = lane; j < D; j += 32) {
        float v = xr[j];
        if (KIND == ROW_CATEGORICAL) v = gumbel_val(v, sd, salt, r * D + j);
        if (bi == 0x7fffffff || v > best) { best = v; bi = (int)j; }
      }
      warp_argmax(best, bi);
      if (lane == 0) reinterpret_cast<int*>(out)[r] = bi == 0x7fffffff ? 0 : bi;
    } else {
      int64_t lim = (KIND == ROW_SOFTMAX_CAUSAL) ? (r % D) + 1 : D;
      float m = -INFINITY, s = 0.f;
      for (int64_t j = lane; j < lim; j += 32) {
        float v = xr[j];
        if (v > m) { s = (m == -INFINITY) ? 0.f : s * expf(m - v); m = v; }
        s += expf(v - m);
      }
      warp_online(m, s);
      float* o = reinterpret_cast<float*>(out) + r * D;
      if (KIND == ROW_LOGSOFTMAX) {
        float lz = m + logf(s);
        for (int64_t j = lane; j < D; j += 32) o[j] = xr[j] - lz;
      } else {
        for (int64_t j = lane; j < D; j += 32) o[j] = j < lim ? __fdiv_rn(expf(xr[j] - m), s) : 0.f;
      }
    }
  }
}

template <int KIND>
__global__ void __launch_bounds__(256) row_block_kernel(const float* __restrict__ x, void* __restrict__ out,
                                                        int64_t rows, int64_t D, const int* seed, uint32_t salt) {
  __shared__ float sm_a[8];
  __shared__ float sm_b[8];
  __shared__ int sm_i[8];
  int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  // rows of whole float4s from a 16-byte aligned base (log-softmax over a vocabulary)
  const bool vec4 = KIND == ROW_LOGSOFTMAX && (D & 3) == 0 && !(reinterpret_cast<uintptr_t>(x) & 15) &&
                    !(reinterpret_cast<uintptr_t>(out) & 15);
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* xr = x + r * D;
    if (KIND == ROW_SUM || KIND == ROW_MEAN) {
      float s = 0.f;
      for (int64_t j = threadIdx.x; j < D; j += blockDim.x) s += xr[j];
      s = warp_sum(s);
      if (lane == 0) sm_a[wid] = s;
      __syncthreads();
      if (wid == 0) {
        s = lane < 8 ? sm_a[lane] : 0.f;
        s = warp_sum(s);
        if (lane == 0) reinterpret_cast<float*>(out)[r] = KIND == ROW_MEAN ? __fdiv_rn(s, (float)D) : s;
      }
      __syncthreads();
    } else if (KIND == ROW_ARGMAX || KIND == ROW_CATEGORICAL) {
      float best = -INFINITY;
      int bi = 0x7fffffff;
      uint32_t sd = (KIND == ROW_CATEGORICAL && seed) ? (uint32_t)(*seed) : 0u;
      for (int64_t j = threadIdx.x; j < D; j += blockDim.x) {
        float v = xr[j];
        if (KIND == ROW_CATEGORICAL) v = gumbel_val(v, sd, salt, r * D + j);
        if (bi == 0x7fffffff || v > best) { best = v; bi = (int)j; }
      }
      warp_argmax(best, bi);
      if (lane == 0) { sm_a[wid] = best; sm_i[wid] = bi; }
      __syncthreads();
      if (wid == 0) {
        best = lane < 8 ? sm_a[lane] : -INFINITY;
        bi = lane < 8 ? sm_i[lane] : 0x7fffffff;
        warp_argmax(best, bi);
        if (lane == 0) reinterpret_cast<int*>(out)[r] = bi == 0x7fffffff ? 0 : bi;
      }
      __syncthreads();
    } else {
      int64_t lim = (KIND == ROW_SOFTMAX_CAUSAL) ? (r % D) + 1 : D;
      float m = -INFINITY, s = 0.f;
      int64_t j0 = 0;
      if (vec4) {
        // four elements per step: one rescale per float4, then their exps
        const int64_t n4 = lim >> 2;
        const float4* x4 = reinterpret_cast<const float4*>(xr);
        for (int64_t q = threadIdx.x; q < n4; q += blockDim.x) {
          const float4 v = __ldg(x4 + q);
          const float lm = fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w));
          if (lm > m) { s = (m == -INFINITY) ? 0.f : s * expf(m - lm); m = lm; }
          s += expf(v.x - m) + expf(v.y - m) + expf(v.z - m) + expf(v.w - m);
        }
        j0 = n4 << 2;
      }
      for (int64_t j = j0 + threadIdx.x; j < lim; j += blockDim.x) {
        float v = xr[j];
        if (v > m) { s = (m == -INFINITY) ? 0.f : s * expf(m - v); m = v; }
        s += expf(v - m);
      }
      warp_online(m, s);
      if (lane == 0) { sm_a[wid] = m; sm_b[wid] = s; }
      __syncthreads();
      if (wid == 0) {
        m = lane < 8 ? sm_a[lane] : -INFINITY;
        s = lane < 8 ? sm_b[lane] : 0.f;
        warp_online(m, s);
        if (lane == 0) { sm_a[0] = m; sm_b[0] = s; }
      }
      __syncthreads();
      m = sm_a[0];
      s = sm_b[0];
      float* o = reinterpret_cast<float*>(out) + r * D;
      if (KIND == ROW_LOGSOFTMAX) {
        float lz = m + logf(s);
        if (vec4) {
          const float4* x4 = reinterpret_cast<const float4*>(xr);
          float4* o4 = reinterpret_cast<float4*>(o);
          for (int64_t q = threadIdx.x; q < (D >> 2); q += blockDim.x) {
            const float4 v = __ldg(x4 + q);
            o4[q] = make_float4(v.x - lz, v.y - lz, v.z - lz, v.w - lz);
          }
        } else {
          for (int64_t j = threadIdx.x; j < D; j += blockDim.x) o[j] = xr[j] - lz;
        }
      } else {
        for (int64_t j = threadIdx.x; j < D; j += blockDim.x) o[j] = j < lim ? __fdiv_rn(expf(xr[j] - m), s) : 0.f;
      }
      __syncthreads();
    }
  }
}

// Long-row sum: partial sums of chunk-sized pieces into scratch.
__global__ void __launch_bounds__(256) row_partial_kernel(const float* __restrict__ x, float* __restrict__ part,
                                                          int64_t rows, int64_t D, int64_t nchunk, int64_t chunk) {
  __shared__ float sm[8];
  int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  for (int64_t w = blockIdx.x; w < rows * nchunk; w += gridDim.x) {
    int64_t r = w / nchunk, c = w % nchunk;
    int64_t j0 = c * chunk, j1 = j0 + chunk < D ? j0 + chunk : D;
    const float* xr = x + r * D;
    float s = 0.f;
    for (int64_t j = j0 + threadIdx.x; j < j1; j += blockDim.x) s += xr[j];
    s = warp_sum(s);
    if (lane == 0) sm[wid] = s;
    __syncthreads();
    if (wid == 0) {
      s = lane < 8 ? sm[lane] : 0.f;
      s = warp_sum(s);
      if (lane == 0) part[w] = s;
    }
    __syncthreads();
  }
}

__global__ void scale_div_kernel(float* v, int64_t n, float d) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) v[i] = __fdiv_rn(v[i], d);
}

template <int KIND>
static void dispatch_row(const float* x, void* out, int64_t rows, int64_t D, cudaStream_t s, const int* seed,
                         uint32_t salt) {
  int sms = device_sm_count();
  if (D <= 2048) {
    int64_t blocks = (rows * 32 + 255) / 256;
    int64_t cap = (int64_t)sms * 16;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    row_warp_kernel<KIND><<<(unsigned)blocks, 256, 0, s>>>(x, out, rows, D, seed, salt);
  } else {
    int64_t blocks = rows < (int64_t)sms * 8 ? rows : (int64_t)sms * 8;
    if (blocks < 1) blocks = 1;
    row_block_kernel<KIND><<<(unsigned)blocks, 256, 0, s>>>(x, out, rows, D, seed, salt);
  }
}

// Number of chunk partials used for the long-row path; <= 1 means unused.
static int64_t long_row_chunks(int64_t rows, int64_t D) {
  int sms = device_sm_count();
  if (rows >= sms || D < (1 << 15)) return 0;
  int64_t want = ((int64_t)sms * 4 + rows - 1) / rows;
  int64_t byD = D / 4096;
  return want < byD ? want : byD;
}

size_t row_scratch_floats(int kind, int64_t rows, int64_t D) {
  if (kind != ROW_SUM && kind != ROW_MEAN) return 0;
  int64_t c = long_row_chunks(rows, D);
  return c > 1 ? (size_t)(rows * c) : 0;
}

// Softmax / logSoftmax of rows up to 32*NV long with the row held in
// registers: one load, a warp max, one exp per element, a warp sum, one
// store (element j of the row lives in lane j % 32, slot j / 32, so every
// load and store is a coalesced 128-byte warp access).
__device__ __forceinline__ uint32_t pcg_s(uint32_t h) {
  h = h * 747796405u + 2891336453u;
  h = ((h >> ((h >> 28u) + 4u)) ^ h) * 277803737u;
  return (h >> 22u) ^ h;
}

template <int KIND, int NV, bool DROP = false>
__global__ void __launch_bounds__(256) row_softmax_reg_kernel(const float* __restrict__ x, float* __restrict__ out,
                                                              int64_t rows, int64_t D,
                                                              const __grid_constant__ RowDropout drop = RowDropout{}) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t r = warp; r < rows; r += nwarps) {
    const float* xr = x + r * D;
    const int64_t lim = (KIND == ROW_SOFTMAX_CAUSAL) ? (r % D) + 1 : D;
    float v[NV];
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int64_t j = lane + 32 * i;
      v[i] = j < lim ? __ldg(xr + j) : -INFINITY;
      m = fmaxf(m, v[i]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int64_t j = lane + 32 * i;
      const float e = j < lim ? expf(v[i] - m) : 0.f;
      if (KIND == ROW_SOFTMAX_CAUSAL) v[i] = e;
      sum += e;
    }
    sum = warp_sum(sum);
    float* o = out + r * D;
    if (KIND == ROW_LOGSOFTMAX) {
      const float lz = m + logf(sum);
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const int64_t j = lane + 32 * i;
        if (j < D) o[j] = v[i] - lz;
      }
    } else {
      const uint32_t seed = DROP && drop.seed ? (uint32_t)(*drop.seed) : 0u;
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const int64_t j = lane + 32 * i;
        if (j < D) {
          const float pv = j < lim ? __fdiv_rn(v[i], sum) : 0.f;
          o[j] = pv;
          if (DROP) {
            const uint32_t hsh = pcg_s(seed ^ drop.salt ^ (uint32_t)(drop.drop_off + r * D + j));
            const float u = __uint2float_rn(hsh) * 2.3283064365386963e-10f;  // exact divide by 2^32
            drop.out2[r * D + j] = __fmul_rn(pv, u >= drop.p ? drop.keep_scale : 0.f);
          }
        }
      }
    }
  }
}

template <int KIND>
static bool launch_softmax_reg(const float* x, float* out, int64_t rows, int64_t D, cudaStream_t s) {
  int64_t warps_per_block = 8, blocks = (rows + warps_per_block - 1) / warps_per_block;
  const int64_t cap = (int64_t)device_sm_count() * 16;
  const unsigned g = (unsigned)(blocks < cap ? blocks : cap);
  if (D <= 32) row_softmax_reg_kernel<KIND, 1><<<g, 256, 0, s>>>(x, out, rows, D);
  else if (D <= 64) row_softmax_reg_kernel<KIND, 2><<<g, 256, 0, s>>>(x, out, rows, D);
  else if (D <= 128) row_softmax_reg_kernel<KIND, 4><<<g, 256, 0, s>>>(x, out, rows, D);
  else if (D <= 256) row_softmax_reg_kernel<KIND, 8><<<g, 256, 0, s>>>(x, out, rows, D);
  else if (D <= 512) row_softmax_reg_kernel<KIND, 16><<<g, 256, 0, s>>>(x, out, rows, D);
  else if (D <= 1024) row_softmax_reg_kernel<KIND, 32><<<g, 256, 0, s>>>(x, out, rows, D);
  else return false;
  return true;
}

bool launch_softmax_causal_dropout(const float* x, float* out, int64_t rows, int64_t D, const RowDropout& d,
                                   cudaStream_t s) {
  if (rows <= 0 || D > 1024) return false;
  const int64_t blocks = (rows + 7) / 8, cap = (int64_t)device_sm_count() * 16;
  const unsigned g = (unsigned)(blocks < cap ? blocks : cap);
  constexpr int K = ROW_SOFTMAX_CAUSAL;
  if (D <= 32) row_softmax_reg_kernel<K, 1, true><<<g, 256, 0, s>>>(x, out, rows, D, d);
  else if (D <= 64) row_softmax_reg_kernel<K, 2, true><<<g, 256, 0, s>>>(x, out, rows, D, d);
  else if (D <= 128) row_softmax_reg_kernel<K, 4, true><<<g, 256, 0, s>>>(x, out, rows, D, d);
  else if (D <= 256) row_softmax_reg_kernel<K, 8, true><<<g, 256, 0, s>>>(x, out, rows, D, d);
  else if (D <= 512) row_softmax_reg_kernel<K, 16, true><<<g, 256, 0, s>>>(x, out, rows, D, d);
  else row_softmax_reg_kernel<K, 32, true><<<g, 256, 0, s>>>(x, out, rows, D, d);
  return true;
}

void launch_row(int kind, const float* x, void* out, int64_t rows, int64_t D, cudaStream_t s, const int* seed,
                uint32_t salt, float* scratch, size_t scratch_floats) {
  if (rows <= 0) return;
  if (kind == ROW_SOFTMAX_CAUSAL && launch_softmax_reg<ROW_SOFTMAX_CAUSAL>(x, reinterpret_cast<float*>(out), rows, D, s))
    return;
  if (kind == ROW_LOGSOFTMAX && launch_softmax_reg<ROW_LOGSOFTMAX>(x, reinterpret_cast<float*>(out), rows, D, s))
    return;
  if (kind == ROW_SUM || kind == ROW_MEAN) {
    int64_t c = long_row_chunks(rows, D);
    if (c > 1 && scratch && scratch_floats >= (size_t)(rows * c)) {
      int64_t chunk = (D + c - 1) / c;
      row_partial_kernel<<<(unsigned)(rows * c), 256, 0, s>>>(x, scratch, rows, D, c, chunk);
      dispatch_row<ROW_SUM>(scratch, out, rows, c, s, nullptr, 0);
      // a mean divides the folded sum exactly by D, as the reference does
      if (kind == ROW_MEAN)
        scale_div_kernel<<<(unsigned)((rows + 255) / 256), 256, 0, s>>>(reinterpret_cast<float*>(out), rows,
                                                                         (float)D);
      return;
    }
  }
  switch (kind) {
    case ROW_SUM: dispatch_row<ROW_SUM>(x, out, rows, D, s, seed, salt); break;
    case ROW_MEAN: dispatch_row<ROW_MEAN>(x, out, rows, D, s, seed, salt); break;
    case ROW_ARGMAX: dispatch_row<ROW_ARGMAX>(x, out, rows, D, s, seed, salt); break;
    case ROW_LOGSOFTMAX: dispatch_row<ROW_LOGSOFTMAX>(x, out, rows, D, s, seed, salt); break;
    case ROW_SOFTMAX_CAUSAL: dispatch_row<ROW_SOFTMAX_CAUSAL>(x, out, rows, D, s, seed, salt); break;
    case ROW_CATEGORICAL: dispatch_row<ROW_CATEGORICAL>(x, out, rows, D, s, seed, salt); break;
  }
}

// -------------------------------------------------------------- column sum --
// Column sums run in 256-thread blocks of 32 column threads (one column, or
// four adjacent columns in the float4 form) x 8 row groups: row group g of
// chunk c sums rows r0+g, r0+g+8, ... ascending; the 8 group sums are added
// in group order through shared memory; chunk partials are folded in chunk
// order. The fused column reductions use the same blocks and chunks, so every
// column is summed in the same order whichever kernel runs.
int64_t colsum_col_blocks(int64_t inner, bool vec) {
  const int64_t cols = vec ? (inner + 3) / 4 : inner;
  return (cols + 31) / 32;
}

// Row chunks: at most eight blocks per SM in one wave (column blocks x
// chunks <= 8 x SMs, so no partial second wave), at least 64 rows per chunk.
// Hence chunks x columns <= 8 x SMs x 128 whenever there is more than one.
int64_t colsum_chunks(int64_t outer, int64_t inner) {
  const int64_t sms = device_sm_count();
  const int64_t cb = colsum_col_blocks(inner, inner % 4 == 0);
  const int64_t want = (8 * sms) / cb;
  const int64_t maxc = (outer + 63) / 64;
  const int64_t c = want < maxc ? want : maxc;
  return c < 1 ? 1 : c;
}

size_t colsum_scratch_floats(int64_t outer, int64_t inner) {
  int64_t c = colsum_chunks(outer, inner);
  return c > 1 ? (size_t)(c * inner) : 0;
}

template <bool VEC>
__global__ void __launch_bounds__(256) colsum_partial_kernel(const float* __restrict__ x, float* __restrict__ part,
                                                             int64_t outer, int64_t inner, int64_t rows_per) {
  constexpr int W = VEC ? 4 : 1;
  __shared__ float red[8][32 * W];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int64_t col = ((int64_t)blockIdx.x * 32 + tx) * W;
  const int64_t c = blockIdx.y;
  const int64_t r0 = c * rows_per, r1 = r0 + rows_per < outer ? r0 + rows_per : outer;
  float acc[W];
#pragma unroll
  for (int l = 0; l < W; ++l) acc[l] = 0.f;
  if (col < inner) {
#pragma unroll 8
    for (int64_t r = r0 + ty; r < r1; r += 8) {
      if constexpr (VEC) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(x + r * inner + col));
        acc[0] += v.x; acc[1] += v.y; acc[2] += v.z; acc[3] += v.w;
      } else {
        acc[0] += __ldg(x + r * inner + col);
      }
    }
  }
#pragma unroll
  for (int l = 0; l < W; ++l) red[ty][tx * W + l] = acc[l];
  __syncthreads();
  if (ty == 0 && col < inner) {
#pragma unroll
    for (int l = 0; l < W; ++l) {
      float t = 0.f;
#pragma unroll
      for (int g = 0; g < 8; ++g) t += red[g][tx * W + l];
      part[c * inner + col + l] = t;
    }
  }
}

// 32 columns per block; warp w sums chunks w, w+8, ... (coalesced across the
// warp's 32 columns), then the 8 warp sums are added in warp order. The
// order is fixed, so results are deterministic.
__global__ void __launch_bounds__(256) colsum_fold_kernel(const float* __restrict__ part, float* __restrict__ out,
                                                          int64_t nchunk, int64_t inner) {
  __shared__ float red[8][33];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t col = (int64_t)blockIdx.x * 32 + lane;
  float s = 0.f;
  if (col < inner) {
    int64_t c = w;
    for (; c + 24 < nchunk; c += 32) {
      const float a = __ldg(part + c * inner + col), b = __ldg(part + (c + 8) * inner + col);
      const float d = __ldg(part + (c + 16) * inner + col), e = __ldg(part + (c + 24) * inner + col);
      s += a; s += b; s += d; s += e;
    }
    for (; c < nchunk; c += 8) s += __ldg(part + c * inner + col);
  }
  red[w][lane] = s;
  __syncthreads();
  if (w == 0 && col < inner) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) t += red[k][lane];
    out[col] = t;
  }
}

void launch_colsum_fold(const float* part, float* out, int64_t nchunk, int64_t inner, cudaStream_t s) {
  colsum_fold_kernel<<<(unsigned)((inner + 31) / 32), 256, 0, s>>>(part, out, nchunk, inner);
}

void launch_colsum(const float* x, float* out, int64_t outer, int64_t inner, float* scratch, cudaStream_t s) {
  if (inner <= 0) return;
  const int64_t c = colsum_chunks(outer, inner);
  const bool chunked = c > 1 && scratch;
  float* dst = chunked ? scratch : out;
  const bool vec = inner % 4 == 0 && !(reinterpret_cast<uintptr_t>(x) & 15);
  const unsigned gx = (unsigned)colsum_col_blocks(inner, vec);
  const int64_t nc = chunked ? c : 1;
  const int64_t rows_per = (outer + nc - 1) / nc;
  if (vec)
    colsum_partial_kernel<true><<<dim3(gx, (unsigned)nc), 256, 0, s>>>(x, dst, outer, inner, rows_per);
  else
    colsum_partial_kernel<false><<<dim3(gx, (unsigned)nc), 256, 0, s>>>(x, dst, outer, inner, rows_per);
  if (chunked) launch_colsum_fold(scratch, out, nc, inner, s);
}

// ---------------------------------------------------- general sum to shape --
struct SumGen {
  int rank;
  int64_t in_dims[8];
  int64_t in_strides[8];
  int64_t keep[8];
  int64_t out_dims[8];
  int64_t red_count;
};

__global__ void __launch_bounds__(256) sum_general_kernel(const float* __restrict__ x, float* __restrict__ out,
                                                          const __grid_constant__ SumGen g, int64_t out_numel) {
  __shared__ float sm[8];
  int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  for (int64_t o = blockIdx.x; o < out_numel; o += gridDim.x) {
    int64_t base = 0, rem = o;
    for (int d = g.rank - 1; d >= 0; --d) {
      int64_t c = rem % g.out_dims[d];
      rem /= g.out_dims[d];
      if (g.keep[d]) base += c * g.in_strides[d];
    }
    float s = 0.f;
    for (int64_t k = threadIdx.x; k < g.red_count; k += blockDim.x) {
      int64_t off = base, rr = k;
      for (int d = g.rank - 1; d >= 0; --d) {
        if (g.keep[d]) continue;
        int64_t c = rr % g.in_dims[d];
        rr /= g.in_dims[d];
        off += c * g.in_strides[d];
      }
      s += x[off];
    }
    s = warp_sum(s);
    if (lane == 0) sm[wid] = s;
    __syncthreads();
    if (wid == 0) {
      s = lane < 8 ? sm[lane] : 0.f;
      s = warp_sum(s);
      if (lane == 0) out[o] = s;
    }
    __syncthreads();
  }
}

// ------------------------------------------------ middle-axis sum [R1,K,R2] --
// out[c] = sum over b < R1, i < R2 of x[(b*K + c)*R2 + i] (a conv bias
// gradient: batch and spatial axes reduced, channels kept). Block (c, s) sums
// the batch slice s of channel c reading contiguous R2-runs; partials
// part[s*K + c] are then folded over s in order, so the result does not
// depend on scheduling.
static int64_t sum_mid_slices(int64_t R1, int64_t K) {
  int64_t s = (4 * (int64_t)device_sm_count() + K - 1) / K;
  if (s > R1) s = R1;
  if (s > 64) s = 64;
  return s < 1 ? 1 : s;
}

int64_t sum_mid_scratch_floats(int64_t R1, int64_t K) { return sum_mid_slices(R1, K) * K; }

__global__ void __launch_bounds__(256) sum_mid_partial_kernel(const float* __restrict__ x, float* __restrict__ part,
                                                              int64_t R1, int64_t K, int64_t R2, int64_t per) {
  __shared__ float sm[8];
  const int64_t c = blockIdx.x, sl = blockIdx.y;
  const int64_t b0 = sl * per, b1 = b0 + per < R1 ? b0 + per : R1;
  float acc = 0.f;
  for (int64_t b = b0; b < b1; ++b) {
    const float* row = x + (b * K + c) * R2;
    for (int64_t i = threadIdx.x; i < R2; i += blockDim.x) acc += row[i];
  }
  acc = warp_sum(acc);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) sm[wid] = acc;
  __syncthreads();
  if (wid == 0) {
    acc = lane < 8 ? sm[lane] : 0.f;
    acc = warp_sum(acc);
    if (lane == 0) part[sl * K + c] = acc;
  }
}

void launch_sum_mid(const float* x, float* out, int64_t R1, int64_t K, int64_t R2, float* scratch, cudaStream_t s) {
  const int64_t S = sum_mid_slices(R1, K);
  const int64_t per = (R1 + S - 1) / S;
  const int64_t used = (R1 + per - 1) / per;
  sum_mid_partial_kernel<<<dim3((unsigned)K, (unsigned)used), 256, 0, s>>>(x, scratch, R1, K, R2, per);
  launch_colsum_fold(scratch, out, used, K, s);
}

void launch_sum_general(const float* x, float* out, int rank, const int64_t* in_dims, const int64_t* keep,
                        int64_t in_numel, int64_t out_numel, cudaStream_t s) {
  SumGen g{};
  g.rank = rank;
  int64_t st = 1;
  for (int d = rank - 1; d >= 0; --d) {
    g.in_dims[d] = in_dims[d];
    g.in_strides[d] = st;
    st *= in_dims[d];
    g.keep[d] = keep[d];
    g.out_dims[d] = keep[d] ? in_dims[d] : 1;
  }
  g.red_count = out_numel > 0 ? in_numel / out_numel : 0;
  int64_t cap = (int64_t)device_sm_count() * 16;
  int64_t blocks = out_numel < cap ? out_numel : cap;
  if (blocks < 1) return;
  sum_general_kernel<<<(unsigned)blocks, 256, 0, s>>>(x, out, g, out_numel);
}

}  // namespace tg
