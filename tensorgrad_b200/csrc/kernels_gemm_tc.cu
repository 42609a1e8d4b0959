// f32 GEMM on the 5th-generation tensor cores with a 3xTF32 split.
//
// Replaces the reference's matmul / matmul_batched kernels
// (src/codegen.ts:496-601, 16x16 shared-memory tiles of scalar f32 FMA) for
// every contraction whose operands TMA can describe.
//
// Accuracy: each f32 operand x is split into hi = x with the low 13 mantissa
// bits cleared (exactly representable in TF32) and lo = x - hi (exact in
// f32, then truncated to TF32 by the tensor core). The product is
// accumulated as lo_a*hi_b + hi_a*lo_b + hi_a*hi_b in one f32 TMEM
// accumulator; the dropped lo_a*lo_b term and the truncation of lo are
// ~2^-20 relative, so results match an f32 GEMM to ~1e-6.
//
// Structure (one CTA per 128x128 output tile, 192 threads):
//   warp 0     TMA producer: per 32-deep K stage loads the A and B tiles
//              (128B-swizzled; K-major: one 128x32 box; MN-major: sixteen
//              8(K)x32(MN) boxes in UMMA's canonical MN-major atom order)
//              into a 3-stage ring
//   warp 1     allocates TMEM (128 f32 columns), issues the tcgen05.mma
//              instructions (M=128, N=128, K=8, kind::tf32) from one thread,
//              commits each stage back to the producer
//   warps 2-5  split each landed stage into K-major hi and lo tiles (in
//              place for K-major operands; transposed out of a staging box for
//              MN-major ones), drain finished accumulator chunks into f32
//              registers, then store alpha*acc (+bias) (+C)
// Every mbarrier wait is bounded; on timeout the kernel records an error
// code in g_gemm_tc_error and leaves without further waits.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdio>
#include <cstring>

#include "kernels.cuh"

namespace tg {

__device__ int g_gemm_tc_error = 0;
// Progress markers of CTA (0,0,0) for diagnosing a stalled pipeline:
// [0] producer stages issued, [1] stages split, [2] MMA stages issued,
// [3] epilogue reached.
__device__ int g_gemm_tc_dbg[8];

constexpr int TC_BM = 128, TC_BN = 128, TC_BK = 32, TC_STAGES = 2;
constexpr int TC_TILE_BYTES = 128 * TC_BK * 4;           // 16 KB per operand tile
// A_hi, B_hi, A_lo, B_lo (K-major, what the MMA reads) + A/B staging for
// MN-major operands (what TMA writes when the operand is not K-major)
constexpr int TC_STAGE_BYTES = 6 * TC_TILE_BYTES;
constexpr int TC_SMEM = TC_STAGES * TC_STAGE_BYTES + 1024 + 256;
constexpr uint32_t TC_TMEM_COLS = 256;  // two 128-column accumulators
constexpr long long TC_SPIN_LIMIT = 1ll << 22;

struct TcParams {
  int64_t M, N, K;
  int64_t batch, batch2;
  int a_kmajor, b_kmajor;
  int a_b1, a_b2, b_b1, b_b2;  // 1 when that operand varies with the batch index
  float* C;
  int64_t ldc, c_batch, c_batch2;
  const float* bias;
  float alpha;
  int accumulate;
  int splits, kps;  // split-K: number of K ranges and K-stages per range
  float* ws;        // [splits][batch][M][N] partial tiles when splits > 1
};

// ------------------------------------------------------------- PTX helpers --
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok) : "r"(smem_u32(b)), "r"(parity) : "memory");
  return ok != 0;
}
// Bounded wait: false (and an error code recorded) after TC_SPIN_LIMIT tries.
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, int code) {
  for (long long i = 0; i < TC_SPIN_LIMIT; ++i)
    if (mbar_try(b, parity)) return true;
  atomicExch(&g_gemm_tc_error, code);
  return false;
}
__device__ __forceinline__ void tma_load_4d(const CUtensorMap* tm, uint64_t* bar, void* dst, int c0, int c1, int c2,
                                            int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];"
      ::"r"(smem_u32(dst)), "l"(tm), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for sm_100
  d |= (uint64_t)2 << 61;  // 128-byte swizzle
  return d;
}
__device__ __forceinline__ void umma_tf32(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
  // The disable-output-lane mask is given explicitly (all lanes enabled).
  const uint32_t z = 0;
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n"
      ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(acc), "r"(z), "r"(z), "r"(z), "r"(z));
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// ------------------------------------------------------------------ kernel --
// Accumulator chunking: the tensor core accumulates in f32 without
// round-to-nearest on every add, so error grows with the number of
// accumulation steps. The MMA warp therefore alternates between two TMEM
// accumulators every TC_CHUNK K-stages (384 MMA-K), and the split/epilogue
// warps drain each finished accumulator into per-thread f32 registers with
// round-to-nearest adds; total error then grows like sqrt(K) instead of K.
constexpr int TC_CHUNK = 4;

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// Split one landed stage (both operands) into K-major hi/lo tiles.
__device__ __forceinline__ void split_stage(uint8_t* st, int t, int a_kmajor, int b_kmajor) {
#pragma unroll 1
  for (int op = 0; op < 2; ++op) {
    const bool kmaj = op == 0 ? a_kmajor : b_kmajor;
    uint8_t* hi_t = st + op * TC_TILE_BYTES;
    uint8_t* lo_t = st + (2 + op) * TC_TILE_BYTES;
    if (kmaj) {
      // landed K-major: split in place, lo into the twin buffer (same layout)
      float4* hi = reinterpret_cast<float4*>(hi_t);
      float4* lo = reinterpret_cast<float4*>(lo_t);
#pragma unroll 4
      for (int q = t; q < TC_TILE_BYTES / 16; q += 128) {
        float4 x = hi[q], h, l;
        const float* xv = &x.x;
        float* hv = &h.x;
        float* lv = &l.x;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float hh = __uint_as_float(__float_as_uint(xv[e]) & 0xFFFFE000u);
          hv[e] = hh;
          lv[e] = xv[e] - hh;
        }
        hi[q] = h;
        lo[q] = l;
      }
    } else {
      // landed MN-major in staging: 4 boxes (MN chunk j) of 32 K-rows x
      // 128 bytes; element (k, mn) sits in row k, 16-byte chunk
      // (mn%32)/4 XOR (k%8). Write hi/lo transposed into the K-major
      // tiles: element (mn, k) in row mn, chunk (k/4) XOR (mn%8).
      const uint8_t* stg = st + (4 + op) * TC_TILE_BYTES;
#pragma unroll 2
      for (int q = t; q < TC_TILE_BYTES / 16; q += 128) {
        const int j = q >> 8;
        const int k = (q >> 3) & 31;
        const int pc = q & 7;
        const int lc = pc ^ (k & 7);
        const float4 x = *reinterpret_cast<const float4*>(stg + q * 16);
        const float* xv = &x.x;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int mn = j * 32 + lc * 4 + e;
          const uint32_t o = (uint32_t)mn * 128u + (uint32_t)((((k >> 2) ^ (mn & 7)) << 4) + ((k & 3) << 2));
          const float hh = __uint_as_float(__float_as_uint(xv[e]) & 0xFFFFE000u);
          *reinterpret_cast<float*>(hi_t + o) = hh;
          *reinterpret_cast<float*>(lo_t + o) = xv[e] - hh;
        }
      }
    }
  }
}

__global__ void __launch_bounds__(192, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA,
                                                         const __grid_constant__ CUtensorMap tmB,
                                                         const __grid_constant__ TcParams P) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + TC_STAGES * TC_STAGE_BYTES);
  uint64_t* conv = full + TC_STAGES;
  uint64_t* empty = conv + TC_STAGES;
  uint64_t* dfull = empty + TC_STAGES;   // [2] accumulator chunk finished (MMA commit)
  uint64_t* dempty = dfull + 2;          // [2] accumulator drained (128 epilogue threads)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(dempty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n0 = (int64_t)blockIdx.x * TC_BN, m0 = (int64_t)blockIdx.y * TC_BM;
  const int64_t zb = blockIdx.z / P.splits;   // batch index
  const int sp = blockIdx.z % P.splits;       // K range
  const int i1 = (int)(zb / P.batch2), i2 = (int)(zb % P.batch2);
  const int nk_all = (int)((P.K + TC_BK - 1) / TC_BK);
  const int kbeg = sp * P.kps;
  const int nk = max(0, min(nk_all, kbeg + P.kps) - kbeg);
  const int nchunks = (nk + TC_CHUNK - 1) / TC_CHUNK;
  const bool first_cta = blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0;
  const bool partial = P.splits > 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < TC_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], 128);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&dfull[a], 1);
      mbar_init(&dempty[a], 128);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TC_TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == 0) {
    // ---------------------------------------------------------- producer --
    if (lane == 0) {
      const int ab1 = P.a_b1 ? i1 : 0, ab2 = P.a_b2 ? i2 : 0;
      const int bb1 = P.b_b1 ? i1 : 0, bb2 = P.b_b2 ? i2 : 0;
      for (int it = 0; it < nk && ok; ++it) {
        const int s = it % TC_STAGES;
        const uint32_t ph = (uint32_t)(it / TC_STAGES) & 1u;
        if (it >= TC_STAGES && !mbar_wait(&empty[s], ph ^ 1u, 1)) { ok = false; break; }
        uint8_t* st = smem + s * TC_STAGE_BYTES;
        mbar_expect_tx(&full[s], 2 * TC_TILE_BYTES);
        const int k0 = (kbeg + it) * TC_BK;
        if (P.a_kmajor) tma_load_4d(&tmA, &full[s], st, k0, (int)m0, ab1, ab2);
        else for (int j = 0; j < 4; ++j)
          tma_load_4d(&tmA, &full[s], st + 4 * TC_TILE_BYTES + j * 4096, (int)m0 + 32 * j, k0, ab1, ab2);
        if (P.b_kmajor) tma_load_4d(&tmB, &full[s], st + TC_TILE_BYTES, k0, (int)n0, bb1, bb2);
        else for (int j = 0; j < 4; ++j)
          tma_load_4d(&tmB, &full[s], st + 5 * TC_TILE_BYTES + j * 4096, (int)n0 + 32 * j, k0, bb1, bb2);
        if (first_cta) g_gemm_tc_dbg[0] = it + 1;
      }
    }
  } else if (warp == 1) {
    // --------------------------------------------------------------- MMA --
    if (lane == 0) {
      // kind::tf32 instruction descriptor: D f32, A/B tf32, K-major, N>>3, M>>4
      const uint32_t idesc = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(TC_BN >> 3) << 17) |
                             ((uint32_t)(TC_BM >> 4) << 24);
      for (int it = 0; it < nk && ok; ++it) {
        const int s = it % TC_STAGES;
        const uint32_t ph = (uint32_t)(it / TC_STAGES) & 1u;
        const int chunk = it / TC_CHUNK, acc = chunk & 1;
        const bool chunk_start = (it % TC_CHUNK) == 0;
        if (chunk_start && chunk >= 2 && !mbar_wait(&dempty[acc], (uint32_t)((chunk - 2) >> 1) & 1u, 5)) {
          ok = false; break;
        }
        if (!mbar_wait(&conv[s], ph, 2)) { ok = false; break; }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t base = smem_u32(smem + s * TC_STAGE_BYTES);
        const uint32_t a_hi = base, b_hi = base + TC_TILE_BYTES;
        const uint32_t a_lo = base + 2 * TC_TILE_BYTES, b_lo = base + 3 * TC_TILE_BYTES;
        const uint32_t dacc = tmem + (uint32_t)(acc * TC_BN);
#pragma unroll
        for (int kk = 0; kk < TC_BK / 8; ++kk) {
          // K-major tiles: 128 rows of 128 bytes (32 K values), 8-row groups
          // 1 KB apart (SBO); a K step of 8 advances 32 bytes in the row.
          const uint32_t off = kk * 32;
          uint64_t dAh = umma_desc(a_hi + off, 16, 1024), dAl = umma_desc(a_lo + off, 16, 1024);
          uint64_t dBh = umma_desc(b_hi + off, 16, 1024), dBl = umma_desc(b_lo + off, 16, 1024);
          const uint32_t first = (chunk_start && kk == 0) ? 0u : 1u;
          umma_tf32(dacc, dAl, dBh, idesc, first);
          umma_tf32(dacc, dAh, dBl, idesc, 1u);
          umma_tf32(dacc, dAh, dBh, idesc, 1u);
        }
        umma_commit(&empty[s]);  // frees the stage once these MMAs have read it
        if ((it % TC_CHUNK) == TC_CHUNK - 1 || it == nk - 1) umma_commit(&dfull[acc]);
        if (first_cta) g_gemm_tc_dbg[2] = it + 1;
      }
    }
  } else {
    // ---------------------------------------- split, drain, then epilogue --
    const int t = threadIdx.x - 64;  // 0..127
    const int g = warp & 3;          // TMEM lane group this warp may access
    float sum[TC_BN];
#pragma unroll
    for (int j = 0; j < TC_BN; ++j) sum[j] = 0.f;
    int drained = 0;
    auto drain = [&](int c) -> bool {
      const int acc = c & 1;
      if (!mbar_wait(&dfull[acc], (uint32_t)(c >> 1) & 1u, 4)) return false;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
      for (int q = 0; q < TC_BN / 32; ++q) {
        uint32_t r[32];
        tmem_ld32(tmem + ((uint32_t)(g * 32) << 16) + (uint32_t)(acc * TC_BN + q * 32), r);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
        for (int j = 0; j < 32; ++j) sum[q * 32 + j] += __uint_as_float(r[j]);
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      mbar_arrive(&dempty[acc]);
      return true;
    };
    for (int it = 0; it < nk && ok; ++it) {
      const int s = it % TC_STAGES;
      const uint32_t ph = (uint32_t)(it / TC_STAGES) & 1u;
      if (!mbar_wait(&full[s], ph, 3)) { ok = false; break; }
      uint8_t* st = smem + s * TC_STAGE_BYTES;
      split_stage(st, t, P.a_kmajor, P.b_kmajor);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive(&conv[s]);
      if (t == 0 && first_cta) g_gemm_tc_dbg[1] = it + 1;
      // after splitting the last stage of chunk c+1, drain chunk c
      if ((it % TC_CHUNK) == TC_CHUNK - 1 && it / TC_CHUNK >= 1) {
        if (!drain(drained)) { ok = false; break; }
        ++drained;
      }
    }
    while (ok && drained < nchunks) {
      if (!drain(drained)) { ok = false; break; }
      ++drained;
    }
    if (ok) {
      if (t == 0 && first_cta) g_gemm_tc_dbg[3] = 1;
      const int64_t row = m0 + g * 32 + lane;
      // split-K: raw partial tile into the workspace, finished by gemm_splitk_reduce
      float* C = partial ? P.ws + ((int64_t)sp * P.batch + zb) * P.M * P.N
                         : P.C + (int64_t)i1 * P.c_batch + (int64_t)i2 * P.c_batch2;
      const int64_t ldc = partial ? P.N : P.ldc;
      const float alpha = partial ? 1.f : P.alpha;
      const float* bias = partial ? nullptr : P.bias;
      const int accumulate = partial ? 0 : P.accumulate;
      if (row < P.M) {
#pragma unroll
        for (int q = 0; q < TC_BN / 32; ++q) {
          const int64_t col0 = n0 + q * 32;
          if (col0 >= P.N) break;
          float* dst = C + row * ldc + col0;
          const bool vec = (col0 + 32 <= P.N) && ((ldc & 3) == 0) &&
                           ((reinterpret_cast<uintptr_t>(dst) & 15) == 0);
          if (vec) {
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
              float4 v = make_float4(sum[q * 32 + j] * alpha, sum[q * 32 + j + 1] * alpha,
                                     sum[q * 32 + j + 2] * alpha, sum[q * 32 + j + 3] * alpha);
              if (bias) {
                v.x += bias[col0 + j]; v.y += bias[col0 + j + 1];
                v.z += bias[col0 + j + 2]; v.w += bias[col0 + j + 3];
              }
              float4* d4 = reinterpret_cast<float4*>(dst + j);
              if (accumulate) {
                float4 o = *d4;
                v.x += o.x; v.y += o.y; v.z += o.z; v.w += o.w;
              }
              *d4 = v;
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              if (col0 + j < P.N) {
                float v = sum[q * 32 + j] * alpha;
                if (bias) v += bias[col0 + j];
                if (accumulate) v += dst[j];
                dst[j] = v;
              }
            }
          }
        }
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TC_TMEM_COLS));
  }
}

// Deterministic split-K reduction: C = alpha * sum_sp ws[sp] (+bias) (+C),
// summed in split order.
__global__ void __launch_bounds__(256) gemm_splitk_reduce(const __grid_constant__ TcParams P) {
  const int64_t per = P.M * P.N;
  const int64_t total = per * P.batch;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += stride) {
    const int64_t zb = e / per, rem = e % per, row = rem / P.N, col = rem % P.N;
    float v = 0.f;
    for (int sp = 0; sp < P.splits; ++sp) v += P.ws[(int64_t)sp * total + e];
    v *= P.alpha;
    if (P.bias) v += P.bias[col];
    const int64_t i1 = zb / P.batch2, i2 = zb % P.batch2;
    float* d = P.C + i1 * P.c_batch + i2 * P.c_batch2 + row * P.ldc + col;
    *d = P.accumulate ? *d + v : v;
  }
}

// ------------------------------------------------------------------- host --
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// Tensor map for one operand. kmajor: dims {K, MN, b1, b2}; else {MN, K, b1, b2}.
static bool make_map(CUtensorMap* tm, const float* base, bool kmajor, int64_t mn, int64_t k, int64_t ld_mn,
                     int64_t ld_k, int64_t e1, int64_t s1, int64_t e2, int64_t s2) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[4], strides[3];
  cuuint32_t box[4], estr[4] = {1, 1, 1, 1};
  if (kmajor) {
    dims[0] = (cuuint64_t)k; dims[1] = (cuuint64_t)mn; strides[0] = (cuuint64_t)(ld_mn * 4);
    box[0] = TC_BK; box[1] = 128;
  } else {
    dims[0] = (cuuint64_t)mn; dims[1] = (cuuint64_t)k; strides[0] = (cuuint64_t)(ld_k * 4);
    box[0] = 32; box[1] = TC_BK;
  }
  dims[2] = (cuuint64_t)e1; dims[3] = (cuuint64_t)e2;
  strides[1] = (cuuint64_t)((e1 > 1 ? s1 : 1) * 4);
  strides[2] = (cuuint64_t)((e2 > 1 ? s2 : 1) * 4);
  box[2] = 1; box[3] = 1;
  for (int i = 0; i < 3; ++i) {
    if (strides[i] % 16 != 0 || strides[i] == 0) {
      // unit-extent batch dims may use any stride: round it up to a legal value
      if ((i >= 1) && dims[i + 1] == 1) strides[i] = 16;
      else return false;
    }
  }
  CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int gemm_tc_splits(int64_t M, int64_t N, int64_t K, int64_t batch) {
  const int64_t tiles = ((M + TC_BM - 1) / TC_BM) * ((N + TC_BN - 1) / TC_BN) * batch;
  const int64_t nk = (K + TC_BK - 1) / TC_BK;
  const int64_t sms = device_sm_count();
  if (tiles >= sms || nk < 16) return 1;
  int64_t s = (2 * sms) / tiles;        // about two CTAs per SM
  s = s < nk / 8 ? s : nk / 8;          // at least 8 K-stages per split
  s = s < 32 ? s : 32;
  return s < 2 ? 1 : (int)s;
}

int64_t gemm_tc_workspace_floats(int64_t M, int64_t N, int64_t K, int64_t batch) {
  const int s = gemm_tc_splits(M, N, K, batch);
  return s > 1 ? (int64_t)s * batch * M * N : 0;
}

static bool tc_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("TG_GEMM_TC");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

bool launch_gemm_tc(const GemmDesc& g, cudaStream_t s) {
  if (!tc_enabled()) return false;
  // Tiny contractions are cheaper on CUDA cores than a 128x128 tile pipeline.
  if (g.M * g.N * g.K < (int64_t)64 * 64 * 64 || g.K < 16) return false;
  const bool a_k = g.lda_k == 1, a_mn = g.lda_m == 1;
  const bool b_k = g.ldb_k == 1, b_mn = g.ldb_n == 1;
  if (!(a_k || a_mn) || !(b_k || b_mn)) return false;
  if ((reinterpret_cast<uintptr_t>(g.A) & 15) || (reinterpret_cast<uintptr_t>(g.B) & 15)) return false;
  if (g.M > INT32_MAX || g.N > INT32_MAX || g.K > INT32_MAX) return false;
  const int64_t b2 = g.batch2 > 0 ? g.batch2 : 1;
  const int64_t b1 = g.batch / b2;
  CUtensorMap ta, tb;
  const bool ak = a_k;  // prefer K-major when both hold (degenerate dims)
  const bool bk = b_k;
  if (!make_map(&ta, g.A, ak, g.M, g.K, g.lda_m, g.lda_k, g.a_batch ? b1 : 1, g.a_batch, g.a_batch2 ? b2 : 1,
                g.a_batch2))
    return false;
  if (!make_map(&tb, g.B, bk, g.N, g.K, g.ldb_n, g.ldb_k, g.b_batch ? b1 : 1, g.b_batch, g.b_batch2 ? b2 : 1,
                g.b_batch2))
    return false;
  TcParams p{};
  p.M = g.M; p.N = g.N; p.K = g.K;
  p.batch = g.batch; p.batch2 = b2;
  p.a_kmajor = ak ? 1 : 0; p.b_kmajor = bk ? 1 : 0;
  p.a_b1 = g.a_batch ? 1 : 0; p.a_b2 = g.a_batch2 ? 1 : 0;
  p.b_b1 = g.b_batch ? 1 : 0; p.b_b2 = g.b_batch2 ? 1 : 0;
  p.C = g.C; p.ldc = g.ldc; p.c_batch = g.c_batch; p.c_batch2 = g.c_batch2;
  p.bias = g.bias; p.alpha = g.alpha; p.accumulate = g.accumulate;
  const int64_t nk = (g.K + TC_BK - 1) / TC_BK;
  int splits = gemm_tc_splits(g.M, g.N, g.K, g.batch);
  if (splits > 1 && (!g.workspace || g.workspace_floats < (int64_t)splits * g.batch * g.M * g.N)) splits = 1;
  p.kps = (int)((nk + splits - 1) / splits);
  splits = (int)((nk + p.kps - 1) / p.kps);  // every split gets at least one K-stage
  p.splits = splits;
  p.ws = g.workspace;

  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM) != cudaSuccess)
      return false;
    attr = true;
  }
  dim3 grid((unsigned)((g.N + TC_BN - 1) / TC_BN), (unsigned)((g.M + TC_BM - 1) / TC_BM),
            (unsigned)(g.batch * splits));
  gemm_tc_kernel<<<grid, 192, TC_SMEM, s>>>(ta, tb, p);
  if (splits > 1) {
    int64_t total = g.batch * g.M * g.N;
    int64_t blocks = (total + 255) / 256, cap = (int64_t)device_sm_count() * 8;
    gemm_splitk_reduce<<<(unsigned)(blocks < cap ? blocks : cap), 256, 0, s>>>(p);
  }
  return true;
}

int gemm_tc_debug(int* out8) {
  return cudaMemcpyFromSymbol(out8, g_gemm_tc_dbg, 8 * sizeof(int)) == cudaSuccess ? 0 : 1;
}

int gemm_tc_error_flag(bool reset) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_gemm_tc_error, sizeof(int));
  if (reset) {
    int z = 0;
    cudaMemcpyToSymbol(g_gemm_tc_error, &z, sizeof(int));
  }
  return v;
}

}  // namespace tg
