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

__global__ void __launch_bounds__(256) sgemm_kernel(const __grid_constant__ GemmDesc g) {
  __shared__ float As[SG_BK][SG_BM + 4];
  __shared__ float Bs[SG_BK][SG_BN + 4];
  int64_t bz = blockIdx.z;
  int64_t i1 = bz / g.batch2, i2 = bz % g.batch2;
  const float* A = g.A + i1 * g.a_batch + i2 * g.a_batch2;
  const float* B = g.B + i1 * g.b_batch + i2 * g.b_batch2;
  float* C = g.C + i1 * g.c_batch + i2 * g.c_batch2;
  int64_t m0 = (int64_t)blockIdx.y * SG_BM, n0 = (int64_t)blockIdx.x * SG_BN;
  int tid = threadIdx.x;
  int tm = (tid / 16) * 4, tn = (tid % 16) * 4;
  float acc[4][4] = {};
  for (int64_t k0 = 0; k0 < g.K; k0 += SG_BK) {
#pragma unroll
    for (int l = 0; l < 4; ++l) {
      int e = tid + l * 256;
      int mm, kk;
      if (g.lda_k == 1) { mm = e / SG_BK; kk = e % SG_BK; } else { kk = e / SG_BM; mm = e % SG_BM; }
      int64_t gm = m0 + mm, gk = k0 + kk;
      As[kk][mm] = (gm < g.M && gk < g.K) ? A[gm * g.lda_m + gk * g.lda_k] : 0.f;
    }
#pragma unroll
    for (int l = 0; l < 4; ++l) {
      int e = tid + l * 256;
      int nn, kk;
      if (g.ldb_n == 1) { kk = e / SG_BN; nn = e % SG_BN; } else { nn = e / SG_BK; kk = e % SG_BK; }
      int64_t gn = n0 + nn, gk = k0 + kk;
      Bs[kk][nn] = (gn < g.N && gk < g.K) ? B[gk * g.ldb_k + gn * g.ldb_n] : 0.f;
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
      float v = acc[i][j] * g.alpha;
      if (g.bias) v += g.bias[gn];
      float* c = C + gm * g.ldc + gn * (g.ldc_n ? g.ldc_n : 1);
      *c = g.accumulate ? *c + v : v;
    }
  }
}

void launch_gemm_simt(const GemmDesc& g, cudaStream_t s) {
  if (g.M <= 0 || g.N <= 0 || g.batch <= 0) return;
  dim3 grid((unsigned)((g.N + SG_BN - 1) / SG_BN), (unsigned)((g.M + SG_BM - 1) / SG_BM), (unsigned)g.batch);
  sgemm_kernel<<<grid, 256, 0, s>>>(g);
}

}  // namespace tg
