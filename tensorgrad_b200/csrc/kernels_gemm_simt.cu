// General strided batched SGEMM on CUDA cores (f32 FMA, f32 accumulate).
//
// Fallback contraction for shapes/layouts the tcgen05 kernel does not take
// (tiny or oddly strided operands); the reference's WGSL 16x16 tiled kernel
// (src/codegen.ts:1213-1251) is the analogue. 64x64 CTA tile, BK=16, 4x4
// register micro-tile per thread, operands staged through shared memory with
// arbitrary (m,k)/(k,n) strides so permuted views need no copy.
#include "kernels.cuh"

namespace tg {

constexpr int SG_BM = 64, SG_BN = 64, SG_BK = 16;

// splits > 1: blockIdx.z = batch index * splits + K range; each CTA writes a
// raw partial tile to ws[sp][batch][M][N] and sgemm_splitk_reduce finishes.
__global__ void __launch_bounds__(256) sgemm_kernel(const __grid_constant__ GemmDesc g, int splits, int64_t kps) {
  __shared__ float As[SG_BK][SG_BM + 4];
  __shared__ float Bs[SG_BK][SG_BN + 4];
  const int64_t bz = blockIdx.z / splits;
  const int sp = blockIdx.z % splits;
  const int64_t kbeg = sp * kps, kend = kbeg + kps < g.K ? kbeg + kps : g.K;
  int64_t i1 = bz / g.batch2, i2 = bz % g.batch2;
  const float* A = g.A + i1 * g.a_batch + i2 * g.a_batch2;
  const float* B = g.B + i1 * g.b_batch + i2 * g.b_batch2;
  float* C = g.C + i1 * g.c_batch + i2 * g.c_batch2;
  int64_t m0 = (int64_t)blockIdx.y * SG_BM, n0 = (int64_t)blockIdx.x * SG_BN;
  int tid = threadIdx.x;
  int tm = (tid / 16) * 4, tn = (tid % 16) * 4;
  float acc[4][4] = {};
  for (int64_t k0 = kbeg; k0 < kend; k0 += SG_BK) {
#pragma unroll
    for (int l = 0; l < 4; ++l) {
      int e = tid + l * 256;
      int mm, kk;
      if (g.lda_k == 1) { mm = e / SG_BK; kk = e % SG_BK; } else { kk = e / SG_BM; mm = e % SG_BM; }
      int64_t gm = m0 + mm, gk = k0 + kk;
      As[kk][mm] = (gm < g.M && gk < kend) ? A[gm * g.lda_m + gk * g.lda_k] : 0.f;
    }
#pragma unroll
    for (int l = 0; l < 4; ++l) {
      int e = tid + l * 256;
      int nn, kk;
      if (g.ldb_n == 1) { kk = e / SG_BN; nn = e % SG_BN; } else { nn = e / SG_BK; kk = e % SG_BK; }
      int64_t gn = n0 + nn, gk = k0 + kk;
      Bs[kk][nn] = (gn < g.N && gk < kend) ? B[gk * g.ldb_k + gn * g.ldb_n] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < SG_BK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][tm + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tn + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int64_t gm = m0 + tm + i;
    if (gm >= g.M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int64_t gn = n0 + tn + j;
      if (gn >= g.N) continue;
      if (splits > 1) {
        g.workspace[((sp * g.batch + bz) * g.M + gm) * g.N + gn] = acc[i][j];
        continue;
      }
      float v = __fmul_rn(acc[i][j], g.alpha);
      if (g.bias) v += g.bias[gn];
      float* c = C + gm * g.ldc + gn * (g.ldc_n ? g.ldc_n : 1);
      *c = g.accumulate ? *c + v : v;
    }
  }
}

// Deterministic split-K finish: partial tiles summed in split order.
__global__ void __launch_bounds__(256) sgemm_splitk_reduce(const __grid_constant__ GemmDesc g, int splits) {
  const int64_t per = g.M * g.N, total = per * g.batch;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t bz = e / per, rem = e % per, m = rem / g.N, n = rem % g.N;
    float v = 0.f;
    for (int sp = 0; sp < splits; ++sp) v += g.workspace[sp * total + e];
    v = __fmul_rn(v, g.alpha);
    if (g.bias) v += g.bias[n];
    const int64_t i1 = bz / g.batch2, i2 = bz % g.batch2;
    float* c = g.C + i1 * g.c_batch + i2 * g.c_batch2 + m * g.ldc + n * (g.ldc_n ? g.ldc_n : 1);
    *c = g.accumulate ? *c + v : v;
  }
}

void launch_gemm_simt(const GemmDesc& g, cudaStream_t s) {
  if (g.M <= 0 || g.N <= 0 || g.batch <= 0) return;
  const int64_t tiles = ((g.N + SG_BN - 1) / SG_BN) * ((g.M + SG_BM - 1) / SG_BM) * g.batch;
  const int64_t sms = device_sm_count();
  // Few output tiles over a long K: split K across CTAs (up to two per SM),
  // as far as the planner's workspace allows.
  int64_t splits = 1;
  if (tiles < sms && g.K >= 1024 && g.workspace) {
    splits = (2 * sms) / tiles;
    splits = splits < g.K / 256 ? splits : g.K / 256;
    const int64_t fit = g.workspace_floats / (g.batch * g.M * g.N);
    splits = splits < fit ? splits : fit;
    splits = splits < 64 ? splits : 64;
    if (splits < 2) splits = 1;
  }
  int64_t kps = (g.K + splits - 1) / splits;
  kps = (kps + SG_BK - 1) / SG_BK * SG_BK;
  splits = (g.K + kps - 1) / kps;
  dim3 grid((unsigned)((g.N + SG_BN - 1) / SG_BN), (unsigned)((g.M + SG_BM - 1) / SG_BM), (unsigned)(g.batch * splits));
  sgemm_kernel<<<grid, 256, 0, s>>>(g, (int)splits, kps);
  if (splits > 1) {
    const int64_t total = g.batch * g.M * g.N;
    int64_t blocks = (total + 255) / 256, cap = sms * 8;
    sgemm_splitk_reduce<<<(unsigned)(blocks < cap ? blocks : cap), 256, 0, s>>>(g, (int)splits);
  }
}

}  // namespace tg
