// f32 GEMM on the 5th-generation tensor cores with a 3xTF32 split.
//
// Replaces the reference's matmul / matmul_batched kernels
// (src/codegen.ts:496-601, 16x16 shared-memory tiles of scalar f32 FMA) for
// every contraction whose operands TMA can describe.
//
// Accuracy: each f32 operand x is split into hi = x with the low 13 mantissa
// bits cleared (exactly representable in TF32) and lo = x - hi (exact in
// f32, then truncated to TF32 by the tensor core). kind::tf32 MMAs truncate
// their f32 operands (they ignore the low 13 bits; checked on B200), so raw
// f32 data serves as hi without being rewritten. The product is
// accumulated as lo_a*hi_b + hi_a*lo_b + hi_a*hi_b; the dropped lo_a*lo_b
// term and the truncation of lo are ~2^-20 relative.
//
// Data path. A tcgen05 MMA with M=128, N=128, K=8 reads 8 KB of operands in
// 64 clocks when both come from shared memory, which is all of the SM's
// shared-memory bandwidth; three of them per K step plus the split's own
// traffic would leave the tensor pipe idle more than half the time. So only
// B is a shared-memory operand. A goes through tensor memory: the split warps
// read each A row once from the TMA-landed tile, and write its hi and lo
// parts into TMEM with tcgen05.st, and the MMA takes A from TMEM. This also
// makes A's layout free (a K-major or MN-major tile is just read row- or
// column-wise). B must be K-major in shared memory for kind::tf32; the host
// swaps the operands (C^T = B^T A^T) when that puts a K-major operand in B's
// place, and only when neither operand is K-major (weight gradients: both
// are [tokens, features]) do the split warps transpose B.
//
// Structure (one CTA per 128x128 output tile, 192 threads, 3-stage ring):
//   warp 0     TMA producer: per 32-deep K stage, the A tile (K-major: one
//              128x32 box; MN-major: four 32x32 boxes) and the B tile, all
//              128B-swizzled
//   warp 1     allocates all 512 TMEM columns (two 128-column accumulators,
//              then 64 columns of A hi/lo per stage) and issues the MMAs from
//              one thread, committing each stage back to the producer
//   warps 2-5  per stage: A rows -> hi/lo in TMEM, B -> K-major hi/lo tiles
//              in shared memory; drain finished accumulator chunks into f32
//              registers; finally store alpha*acc (+bias) (+C)
// Every mbarrier wait is bounded; on timeout the kernel records an error
// code in g_gemm_tc_error and leaves without further waits.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdio>
#include <cstring>

#include "kernels.cuh"

namespace tg {

__device__ int g_gemm_tc_error = 0;
// Progress markers of CTA 0 for diagnosing a stalled pipeline:
// [0] producer stages issued, [1] stages split, [2] MMA stages issued,
// [3] epilogue reached.
__device__ int g_gemm_tc_dbg[8];
// Pipeline timeline of CTA (0,0,0) when TcParams::trace is set (SM clock
// cycles): [0][it] TMA issued, [1][it] stage landed (split warps),
// [2][it] split done, [3][it] MMAs issued, [4][c] chunk drained,
// [5][0] start, [5][1] epilogue start, [5][2] epilogue end, [6..9][it] each
// split warp done, [10][it] MMA warp saw the stage ready.
constexpr int TC_TRACE_N = 64;
__device__ long long g_gemm_tc_trace[12][TC_TRACE_N];

constexpr int TC_BM = 128, TC_BN = 128, TC_BK = 32;
constexpr int TC_TILE_BYTES = 128 * TC_BK * 4;  // 16 KB per operand tile
// A stage holds `subs` 32-deep K sub-tiles of each operand: [A sub 0..][B hi
// sub 0..] (K-major MMA operand; TMA lands a K-major B here and it is split in
// place) [B lo sub 0..] and, when B is MN-major, [B as landed]. The issuing
// thread's per-stage costs (barrier wait, fence, commits, the bubble before
// the first MMA that reads freshly stored TMEM) are fixed, so large problems
// with a K-major B (many tiles per SM) take 64-deep stages: 24 MMAs each, two
// stages in flight. Otherwise three 32-deep stages: with few tiles per SM the
// deeper ring's shorter fill wins (measured on C4's projections), and an
// MN-major B needs its landing slot.
template <bool BK, int SUBS> struct TcCfg {
  static constexpr int subs = SUBS;
  static constexpr int sk = TC_BK * subs;                 // K per stage
  static constexpr int stages = (BK ? 3 : 4) * SUBS >= 6 ? 2 : 3;
  static constexpr int stage_bytes = (BK ? 3 * subs : 4) * TC_TILE_BYTES;
  static constexpr int epi_tiles = BK && SUBS == 1 ? 4 : 2;  // 32 x 128 output sub-tiles staged at once
  static constexpr int chunk = 4 / subs;  // stages per accumulator chunk: 128 K either way
  static constexpr int ring_bytes = stages * stage_bytes;
  static constexpr int smem = ring_bytes + epi_tiles * TC_TILE_BYTES + 1024 + 256;
};
constexpr uint32_t TC_TMEM_COLS = 512;
constexpr uint32_t TC_ACOL = 2 * TC_BN;  // first TMEM column of the per-stage A hi/lo (64 columns each)
constexpr long long TC_SPIN_LIMIT = 1ll << 22;

struct TcParams {
  int64_t M, N, K;
  int64_t batch, batch2;
  int a_kmajor, b_kmajor;
  int a_b1, a_b2, b_b1, b_b2;  // 1 when that operand varies with the batch index
  float* C;
  int64_t c_m, c_n;            // C(m, n) at C[m*c_m + n*c_n] (c_m == 1 after an operand swap)
  int64_t c_batch, c_batch2;
  const float* bias;
  int bias_m;                  // bias indexed by m (after an operand swap) instead of n
  float alpha;
  int accumulate;
  int splits, kps;  // split-K: number of K ranges and K-stages per range
  float* ws;        // [splits][batch][M][N] partial tiles when splits > 1
  int trace;        // record the pipeline timeline of CTA (0,0,0)
  int tma_store;    // write the tile with TMA stores through tmC (else plain stores)
  int64_t units;    // output tiles x batch x K ranges
  int sk;           // K per pipeline stage (TcCfg::sk of the launched kernel)
  int tri;          // GemmDesc::tri for the output rows (m tiles), or for the columns when
  int tri_n;        // tri_n (the operands were swapped); only without split-K
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
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* tm, const void* src, int c0, int c1, int c2, int c3) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%1, %2, %3, %4}], [%5];"
               ::"l"(tm), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(src))
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
// D (TMEM) (+)= A (TMEM) * B (shared memory descriptor), kind::tf32.
__device__ __forceinline__ void umma_tf32_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t idesc,
                                             uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n}\n"
      ::"r"(tmem_d), "r"(tmem_a), "l"(db), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
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
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// One warp writes 16 consecutive 32-bit columns of its 32 TMEM lanes.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
      ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
        "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

__device__ __forceinline__ float tf32_hi(float x) { return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); }

// ------------------------------------------------------------------ kernel --
// Accumulator chunking: the tensor core accumulates in f32 without
// round-to-nearest on every add, so error grows with the number of
// accumulation steps. The MMA warp therefore alternates between two TMEM
// accumulators every 128 K (TcCfg::chunk stages), and the epilogue warps
// drain each finished accumulator into per-thread f32 registers with
// round-to-nearest adds; total error then grows like sqrt(K) instead of K.

// One output tile of one batch entry and one K range: the persistent CTAs'
// unit of work, numbered with the N tile fastest.
struct TcUnit {
  int64_t m0, n0, zb;
  int sp, i1, i2, kbeg, nk;
};
__device__ __forceinline__ TcUnit tc_unit(const TcParams& P, int64_t u) {
  const int64_t tn = (P.N + TC_BN - 1) / TC_BN, tm = (P.M + TC_BM - 1) / TC_BM;
  const int64_t z = u / (tm * tn), rem = u % (tm * tn);
  TcUnit U;
  U.m0 = (rem / tn) * TC_BM;
  U.n0 = (rem % tn) * TC_BN;
  U.zb = z / P.splits;
  U.sp = (int)(z % P.splits);
  U.i1 = (int)(U.zb / P.batch2);
  U.i2 = (int)(U.zb % P.batch2);
  const int nk_all = (int)((P.K + P.sk - 1) / P.sk);
  U.kbeg = U.sp * P.kps;
  U.nk = max(0, min(nk_all, U.kbeg + P.kps) - U.kbeg);
  if (P.tri) {  // skip the K stages whose products are exactly zero (causal A)
    const int r0 = (int)(P.tri_n ? U.n0 : U.m0);
    if (P.tri == 1) U.nk = min(nk_all, (r0 + TC_BM + P.sk - 1) / P.sk);
    else { U.kbeg = r0 / P.sk; U.nk = max(0, nk_all - U.kbeg); }
  }
  return U;
}

// A tile row r (this thread's TMEM lane) -> hi/lo columns of the stage.
// K-major landing: row r is 128 bytes, 16-byte chunk c stored at c ^ (r % 8).
// MN-major landing: four 32(MN) x 32(K) boxes; element (k, m) of box m / 32
// is in row k at chunk ((m % 32) / 4) ^ (k % 8): a warp reading one k reads
// one 128-byte row, so every access is conflict-free.
__device__ __forceinline__ void split_a_row(const uint8_t* a, int r, bool kmajor, uint32_t tcol) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    float v[16];
    if (kmajor) {
      const uint8_t* row = a + r * 128;
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) {
        const int c = 4 * h + c4;
        const float4 x = *reinterpret_cast<const float4*>(row + ((c ^ (r & 7)) << 4));
        v[4 * c4] = x.x; v[4 * c4 + 1] = x.y; v[4 * c4 + 2] = x.z; v[4 * c4 + 3] = x.w;
      }
    } else {
      const uint8_t* box = a + (r >> 5) * 4096;
      const int m = r & 31;
#pragma unroll
      for (int kk = 0; kk < 16; ++kk) {
        const int k = 16 * h + kk;
        v[kk] = *reinterpret_cast<const float*>(box + k * 128 + ((((m >> 2) ^ (k & 7))) << 4) + ((m & 3) << 2));
      }
    }
    // hi: the raw f32 bits (the MMA truncates them to TF32); lo: the remainder
    uint32_t w[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) w[e] = __float_as_uint(v[e]);
    tmem_st16(tcol + 16 * h, w);
#pragma unroll
    for (int e = 0; e < 16; ++e) w[e] = __float_as_uint(v[e] - tf32_hi(v[e]));
    tmem_st16(tcol + 32 + 16 * h, w);
  }
}

// B tile -> K-major hi and lo tiles, 128 threads. A K-major B landed in
// hi_t; an MN-major one landed in stg.
__device__ __forceinline__ void split_b(uint8_t* hi_t, uint8_t* lo_t, const uint8_t* stg_in, int t, bool kmajor) {
  if (kmajor) {
    // Landed K-major in slot 1, which the MMA reads as hi unchanged: kind::tf32
    // MMAs ignore the low 13 mantissa bits of their f32 operands (truncation,
    // checked on B200), so only lo goes to slot 2 (same layout).
    const float4* raw = reinterpret_cast<const float4*>(hi_t);
    float4* lo = reinterpret_cast<float4*>(lo_t);
#pragma unroll 8
    for (int q = t; q < TC_TILE_BYTES / 16; q += 128) {
      const float4 x = raw[q];
      lo[q] = make_float4(x.x - tf32_hi(x.x), x.y - tf32_hi(x.y), x.z - tf32_hi(x.z), x.w - tf32_hi(x.w));
    }
  } else {
    // Landed MN-major in slot 3: 4 boxes (N chunk j) of 32 K-rows x 128
    // bytes; element (k, n) sits in row k, chunk (n%32)/4 XOR (k%8). Each
    // item is a 4(K) x 4(N) block: four 16-byte row reads, a register
    // transpose, four 16-byte writes each to hi and lo, where element (n, k)
    // sits in row n, chunk (k/4) XOR (n%8). Lanes of a quarter-warp take two
    // N chunks x four K quads: the writes are conflict-free, the reads 2-way.
    const uint8_t* stg = stg_in;
    const int l8 = t & 7, q = (t >> 3) & 3, wq = t >> 5;
#pragma unroll
    for (int it2 = 0; it2 < 2; ++it2) {
      const int R = (wq * 4 + q) * 2 + it2;  // 0..31
      const int c = (R & 3) * 2 + (l8 & 1);
      const int kq = ((R >> 2) & 1) * 4 + (l8 >> 1);
      const int j = R >> 3;
      const uint8_t* box = stg + j * 4096;
      float v[4][4];
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const int k = 4 * kq + kk;
        const float4 x = *reinterpret_cast<const float4*>(box + k * 128 + ((c ^ (k & 7)) << 4));
        v[kk][0] = x.x; v[kk][1] = x.y; v[kk][2] = x.z; v[kk][3] = x.w;
      }
#pragma unroll
      for (int nn = 0; nn < 4; ++nn) {
        const int n = 32 * j + 4 * c + nn;
        const uint32_t o = (uint32_t)n * 128u + (uint32_t)((kq ^ (n & 7)) << 4);
        float4 h, l;
        h.x = tf32_hi(v[0][nn]); h.y = tf32_hi(v[1][nn]); h.z = tf32_hi(v[2][nn]); h.w = tf32_hi(v[3][nn]);
        l.x = v[0][nn] - h.x; l.y = v[1][nn] - h.y; l.z = v[2][nn] - h.z; l.w = v[3][nn] - h.w;
        *reinterpret_cast<float4*>(hi_t + o) = h;
        *reinterpret_cast<float4*>(lo_t + o) = l;
      }
    }
  }
}

// Persistent: each CTA walks units blockIdx.x, blockIdx.x + gridDim.x, ...;
// the stage ring, the accumulator pair and every barrier phase continue
// across units, so one unit's epilogue overlaps the next unit's main loop.
template <bool BK, int SUBS_>
__global__ void __launch_bounds__(448, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA,
                                                         const __grid_constant__ CUtensorMap tmB,
                                                         const __grid_constant__ CUtensorMap tmC,
                                                         const __grid_constant__ TcParams P) {
  constexpr int NS = TcCfg<BK, SUBS_>::stages;
  constexpr int SB = TcCfg<BK, SUBS_>::stage_bytes;
  constexpr int ET = TcCfg<BK, SUBS_>::epi_tiles;
  constexpr int SUBS = SUBS_;
  constexpr int CH = TcCfg<BK, SUBS_>::chunk;
  constexpr int TB = TC_TILE_BYTES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1 KB-aligned base for the 128B-swizzled tiles. Offsetting the shared
  // array (rather than casting through an integer) keeps the pointer in the
  // shared address space, so tile accesses compile to shared loads/stores.
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* epi = smem + TcCfg<BK, SUBS_>::ring_bytes;  // ET output sub-tiles
  uint64_t* full = reinterpret_cast<uint64_t*>(epi + ET * TC_TILE_BYTES);
  uint64_t* conv = full + NS;
  uint64_t* empty = conv + NS;
  uint64_t* dfull = empty + NS;   // [2] accumulator chunk finished (MMA commit)
  uint64_t* dempty = dfull + 2;          // [2] accumulator drained (256 epilogue threads)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(dempty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool partial = P.splits > 1;
  // The pipeline trace exists only in builds with TG_GEMM_TRACE_BUILD
  // defined: the MMA-issuing thread's loop is the kernel's critical path, and
  // even an untaken branch per stage there costs throughput.
#ifdef TG_GEMM_TRACE_BUILD
  const bool tr = P.trace && blockIdx.x == 0;
  auto mark = [&](int row, int i) {
    if (tr && i < TC_TRACE_N) g_gemm_tc_trace[row][i] = clock64();
  };
#else
  auto mark = [](int, int) {};
#endif

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], 128);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&dfull[a], 1);
      mbar_init(&dempty[a], 256);
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
  if (threadIdx.x == 0) mark(5, 0);

  if (warp == 0) {
    // ---------------------------------------------------------- producer --
    if (lane == 0) {
      int gs = 0;
      for (int64_t u = blockIdx.x; u < P.units && ok; u += gridDim.x) {
        const TcUnit U = tc_unit(P, u);
        const int ab1 = P.a_b1 ? U.i1 : 0, ab2 = P.a_b2 ? U.i2 : 0;
        const int bb1 = P.b_b1 ? U.i1 : 0, bb2 = P.b_b2 ? U.i2 : 0;
        for (int it = 0; it < U.nk; ++it, ++gs) {
          const int s = gs % NS;
          const uint32_t ph = (uint32_t)(gs / NS) & 1u;
          if (gs >= NS && !mbar_wait(&empty[s], ph ^ 1u, 1)) { ok = false; break; }
          uint8_t* st = smem + s * SB;
          mark(0, gs);
          if (blockIdx.x == 0) g_gemm_tc_dbg[0] = gs + 1;
          mbar_expect_tx(&full[s], 2 * SUBS * TB);
#pragma unroll
          for (int q = 0; q < SUBS; ++q) {
            const int k0 = (U.kbeg + it) * TcCfg<BK, SUBS_>::sk + TC_BK * q;
            uint8_t* sa = st + q * TB;
            if (P.a_kmajor) tma_load_4d(&tmA, &full[s], sa, k0, (int)U.m0, ab1, ab2);
            else for (int j = 0; j < 4; ++j)
              tma_load_4d(&tmA, &full[s], sa + j * 4096, (int)U.m0 + 32 * j, k0, ab1, ab2);
            if (BK) tma_load_4d(&tmB, &full[s], st + (SUBS + q) * TB, k0, (int)U.n0, bb1, bb2);
            else for (int j = 0; j < 4; ++j)
              tma_load_4d(&tmB, &full[s], st + 3 * TB + j * 4096, (int)U.n0 + 32 * j, k0, bb1, bb2);
          }
        }
      }
    }
  } else if (warp == 1) {
    // --------------------------------------------------------------- MMA --
    if (lane == 0) {
      // kind::tf32 instruction descriptor: D f32, A/B tf32, K-major, N>>3, M>>4
      const uint32_t idesc = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(TC_BN >> 3) << 17) |
                             ((uint32_t)(TC_BM >> 4) << 24);
      // Everything per stage that does not change is computed here: between
      // two stages the issuing thread's work leaves the tensor pipe idle (the
      // MMA queue is about one instruction deep), so the loop keeps only the
      // barrier wait, 12 MMAs and the commits. Shared-memory descriptors
      // advance by address >> 4 in their low field (smem < 256 KB, no carry).
      const uint64_t desc0 = umma_desc(smem_u32(smem) + SUBS * TB, 16, 1024);  // B hi, stage 0, sub 0
      const uint32_t a0 = tmem + TC_ACOL;
      int s = 0, gs = 0;
      uint32_t ph = 0;
      int gc = 0;
      for (int64_t u = blockIdx.x; u < P.units && ok; u += gridDim.x) {
        const TcUnit U = tc_unit(P, u);
        for (int it = 0; it < U.nk; ++it, ++gs) {
          const int c = gc + it / CH, acc = c & 1;
          const bool chunk_start = (it % CH) == 0;
          if (chunk_start && c >= 2 && !mbar_wait(&dempty[acc], (uint32_t)((c - 2) >> 1) & 1u, 5)) {
            ok = false; break;
          }
          if (!mbar_wait(&conv[s], ph, 2)) { ok = false; break; }
          mark(10, gs);
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint64_t dh0 = desc0 + (uint64_t)(s * (SB >> 4));
          const uint32_t a_s = a0 + 64u * SUBS * (uint32_t)s;
          const uint32_t dacc = tmem + (uint32_t)(acc * TC_BN);
#pragma unroll
          for (int q = 0; q < SUBS; ++q) {
            const uint64_t dh = dh0 + (uint64_t)(q * (TB >> 4)), dl = dh + (uint64_t)(SUBS * (TB >> 4));
            const uint32_t a_hi = a_s + 64u * q, a_lo = a_hi + 32u;
#pragma unroll
            for (int kk = 0; kk < TC_BK / 8; ++kk) {
              // B: 128 rows of 128 bytes (32 K values), 8-row groups 1 KB apart
              // (SBO); a K step of 8 advances 32 bytes (2 in the address field).
              // A: 8 TMEM columns.
              const uint32_t first = (chunk_start && q == 0 && kk == 0) ? 0u : 1u;
              umma_tf32_ts(dacc, a_lo + kk * 8, dh + 2 * kk, idesc, first);
              umma_tf32_ts(dacc, a_hi + kk * 8, dl + 2 * kk, idesc, 1u);
              umma_tf32_ts(dacc, a_hi + kk * 8, dh + 2 * kk, idesc, 1u);
            }
          }
          mark(3, gs);
          umma_commit(&empty[s]);  // frees the stage (smem and TMEM A) once these MMAs have read it
          if ((it % CH) == CH - 1 || it == U.nk - 1) umma_commit(&dfull[acc]);
          if (++s == NS) { s = 0; ph ^= 1u; }
        }
        gc += (U.nk + CH - 1) / CH;
      }
    }
  } else if (warp < 6) {
    // ------------------------------------------------------------- split --
    const int t = threadIdx.x - 64;  // 0..127
    const int r = (warp & 3) * 32 + lane;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    // After a failed wait these threads skip the data work but keep the
    // named barrier, so none is left waiting at it.
    int gs = 0;
    for (int64_t u = blockIdx.x; u < P.units; u += gridDim.x) {
      const TcUnit U = tc_unit(P, u);
      for (int it = 0; it < U.nk; ++it, ++gs) {
        const int s = gs % NS;
        const uint32_t ph = (uint32_t)(gs / NS) & 1u;
        if (ok && !mbar_wait(&full[s], ph, 3)) ok = false;
        if (t == 0) mark(1, gs);
        uint8_t* st = smem + s * SB;
        if (ok) {
#pragma unroll
          for (int q = 0; q < SUBS; ++q) {
            split_a_row(st + q * TB, r, P.a_kmajor != 0, tmem + lane_base + TC_ACOL + 64u * (SUBS * (uint32_t)s + q));
            split_b(st + (SUBS + q) * TB, st + (2 * SUBS + q) * TB, st + 3 * TB, t, BK);
          }
        }
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        mbar_arrive(&conv[s]);
        if (t == 0) mark(2, gs);
        if (lane == 0) mark(6 + (t >> 5), gs);
        if (t == 0 && blockIdx.x == 0) g_gemm_tc_dbg[1] = gs + 1;
      }
    }
  } else {
    // ---------------------------------------------------------- epilogue --
    // Eight warps: two per TMEM lane group, each holding 64 of the tile's 128
    // columns in registers. Each finished accumulator chunk is drained and
    // added in f32; the unit's tile is then written in two halves, staged as
    // 128B-swizzled 32 x 128 sub-tiles and stored by TMA (the hardware clips
    // ragged edges). Lines are tile rows for row-major C and tile columns for
    // column-major C. After a failed wait these threads skip the data work but
    // keep every named barrier.
    const int e = threadIdx.x - 192;  // 0..255
    const int r = (warp & 3) * 32 + lane;
    const int hh = (warp - 6) >> 2;   // column half held in registers
    const int cb = 64 * hh;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const float alpha = partial ? 1.f : P.alpha;
    const float* bias = partial ? nullptr : P.bias;
    const bool bias_m = P.bias_m != 0;
    const int64_t cm = partial ? P.N : P.c_m, cn = partial ? 1 : P.c_n;
    const bool colmaj = cm == 1 && cn != 1;
    const bool accumulate = !partial && P.accumulate;
    int gc = 0;
    for (int64_t u = blockIdx.x; u < P.units; u += gridDim.x) {
      const TcUnit U = tc_unit(P, u);
      const int nchunks = (U.nk + CH - 1) / CH;
      float sum[64];
#pragma unroll
      for (int j = 0; j < 64; ++j) sum[j] = 0.f;
      for (int c = 0; c < nchunks; ++c) {
        const int g = gc + c, acc = g & 1;
        if (ok && !mbar_wait(&dfull[acc], (uint32_t)(g >> 1) & 1u, 4)) ok = false;
        if (ok) {
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t v[16];
            tmem_ld16(tmem + lane_base + (uint32_t)(acc * TC_BN + cb + q * 16), v);
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
            for (int j = 0; j < 16; ++j) sum[q * 16 + j] += __uint_as_float(v[j]);
          }
          asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        }
        mbar_arrive(&dempty[acc]);
        if (e == 0) mark(4, g);
      }
      gc += nchunks;
      if (e == 0) mark(5, 1);
      if (e == 0 && blockIdx.x == 0 && ok) g_gemm_tc_dbg[3] += 1;
      float* C = partial ? P.ws + ((int64_t)U.sp * P.batch + U.zb) * P.M * P.N
                         : P.C + (int64_t)U.i1 * P.c_batch + (int64_t)U.i2 * P.c_batch2;
      if (P.tma_store) {
        const float brow = (bias && bias_m && U.m0 + r < P.M) ? bias[U.m0 + r] : 0.f;
        // sub-tile j (0..3) is staged in phase j / ET, in slot j % ET
#pragma unroll
        for (int h = 0; h < 4 / ET; ++h) {
          // the previous TMA store must be done reading the staging buffer
          if (e == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
          asm volatile("bar.sync 2, 256;" ::: "memory");
          if (ok) {
            if (!colmaj) {
              // sub-tile j = tile columns 32j..32j+31, held by the hh == j / 2 warps
#pragma unroll
              for (int jj = 0; jj < 2; ++jj) {
                const int j = 2 * hh + jj;
                if (j / ET != h) continue;
                uint8_t* sub = epi + (j % ET) * TC_TILE_BYTES;
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                  float v[4];
#pragma unroll
                  for (int q = 0; q < 4; ++q) {
                    const int jc = 32 * jj + 4 * c + q;
                    v[q] = __fmul_rn(sum[jc], alpha) + brow;  // alpha rounds alone, as a separate scale would
                    if (bias && !bias_m && U.n0 + cb + jc < P.N) v[q] += bias[U.n0 + cb + jc];
                  }
                  *reinterpret_cast<float4*>(sub + r * 128 + ((c ^ (r & 7)) << 4)) = make_float4(v[0], v[1], v[2], v[3]);
                }
              }
            } else if ((r >> 5) / ET == h) {
              // sub-tile j = tile rows 32j..32j+31, every column line
              uint8_t* sub = epi + ((r >> 5) % ET) * TC_TILE_BYTES + ((r & 3) << 2);
              const int mc = (r & 31) >> 2;
#pragma unroll
              for (int j = 0; j < 64; ++j) {
                const int n = cb + j;
                float v = __fmul_rn(sum[j], alpha) + brow;
                if (bias && !bias_m && U.n0 + n < P.N) v += bias[U.n0 + n];
                *reinterpret_cast<float*>(sub + n * 128 + ((mc ^ (n & 7)) << 4)) = v;
              }
            }
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          asm volatile("bar.sync 2, 256;" ::: "memory");
          if (e == 0 && ok) {
            const int z2 = partial ? U.sp * (int)P.batch + (int)U.zb : U.i1;
            const int z3 = partial ? 0 : U.i2;
            const int64_t inner0 = colmaj ? U.m0 : U.n0, inner_n = colmaj ? P.M : P.N;
            const int outer0 = (int)(colmaj ? U.n0 : U.m0);
#pragma unroll
            for (int sl = 0; sl < ET; ++sl) {
              const int64_t i0 = inner0 + 32 * (h * ET + sl);
              if (i0 < inner_n) tma_store_4d(&tmC, epi + sl * TC_TILE_BYTES, (int)i0, outer0, z2, z3);
            }
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
          }
        }
      } else if (ok) {
        // plain stores: accumulation into C, or a C layout TMA cannot describe
        const int64_t row = U.m0 + r;
        if (row < P.M) {
#pragma unroll
          for (int j = 0; j < 64; ++j) {
            const int64_t col = U.n0 + cb + j;
            if (col < P.N) {
              float v = __fmul_rn(sum[j], alpha);
              if (bias) v += bias[bias_m ? row : col];
              float* d = C + row * cm + col * cn;
              *d = accumulate ? *d + v : v;
            }
          }
        }
      }
      if (e == 0) mark(5, 2);
    }
    if (e == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
  }
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TC_TMEM_COLS));
  }
}

// Deterministic split-K reduction: C = alpha * sum_sp ws[sp] (+bias) (+C),
// summed in split order. Threads walk C's memory order (row-fastest after an
// operand swap) so the stores coalesce; the partial tiles are L2-resident.
__global__ void __launch_bounds__(256) gemm_splitk_reduce(const __grid_constant__ TcParams P) {
  const int64_t per = P.M * P.N;
  const int64_t total = per * P.batch;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const bool rowfast = P.c_m == 1 && P.c_n != 1;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += stride) {
    int64_t zb, row, col;
    if (total <= INT32_MAX) {  // 32-bit index arithmetic (64-bit division is slow)
      const uint32_t e32 = (uint32_t)e, per32 = (uint32_t)per, rem = e32 % per32;
      zb = e32 / per32;
      row = rowfast ? rem % (uint32_t)P.M : rem / (uint32_t)P.N;
      col = rowfast ? rem / (uint32_t)P.M : rem % (uint32_t)P.N;
    } else {
      const int64_t rem = e % per;
      zb = e / per;
      row = rowfast ? rem % P.M : rem / P.N;
      col = rowfast ? rem / P.M : rem % P.N;
    }
    const int64_t w = zb * per + row * P.N + col;
    // partials added in split order; eight loads in flight before their adds
    float v = 0.f;
    int sp = 0;
    for (; sp + 8 <= P.splits; sp += 8) {
      float x[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) x[q] = __ldg(P.ws + (int64_t)(sp + q) * total + w);
#pragma unroll
      for (int q = 0; q < 8; ++q) v += x[q];
    }
    for (; sp < P.splits; ++sp) v += __ldg(P.ws + (int64_t)sp * total + w);
    v = __fmul_rn(v, P.alpha);
    if (P.bias) v += P.bias[P.bias_m ? row : col];
    const int64_t i1 = zb / P.batch2, i2 = zb % P.batch2;
    float* d = P.C + i1 * P.c_batch + i2 * P.c_batch2 + row * P.c_m + col * P.c_n;
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

// Tensor map for one operand. kmajor: dims {K, MN, b1, b2}, box {32, 128};
// else {MN, K, b1, b2}, box {32, 32} (four boxes cover a 128-wide tile).
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
  int64_t s = sms / tiles;              // about one unit per SM
  s = s < nk / 8 ? s : nk / 8;          // at least 8 K-stages per split
  s = s < 128 ? s : 128;                // few-tile, long-K problems (weight gradients) fill the SMs
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
  if ((reinterpret_cast<uintptr_t>(g.A) & 15) || (reinterpret_cast<uintptr_t>(g.B) & 15)) return false;
  if (g.M > INT32_MAX || g.N > INT32_MAX || g.K > INT32_MAX) return false;
  // Operand roles. B must be K-major in shared memory; when only A is,
  // compute C^T = B^T A^T instead (A' = B^T, B' = A^T, C' = C^T).
  const bool swap = g.ldb_k != 1 && g.lda_k == 1;
  int64_t M = g.M, N = g.N;
  const float *A = g.A, *B = g.B;
  int64_t a_m = g.lda_m, a_k = g.lda_k, a_b = g.a_batch, a_b2 = g.a_batch2;
  int64_t b_n = g.ldb_n, b_k = g.ldb_k, b_b = g.b_batch, b_b2 = g.b_batch2;
  int64_t c_m = g.ldc, c_n = g.ldc_n ? g.ldc_n : 1;
  if (swap) {
    std::swap(M, N);
    A = g.B; a_m = g.ldb_n; a_k = g.ldb_k; a_b = g.b_batch; a_b2 = g.b_batch2;
    B = g.A; b_n = g.lda_m; b_k = g.lda_k; b_b = g.a_batch; b_b2 = g.a_batch2;
    std::swap(c_m, c_n);
  }
  const bool ak = a_k == 1, bk = b_k == 1;
  if (!(ak || a_m == 1) || !(bk || b_n == 1)) return false;
  const int64_t b2 = g.batch2 > 0 ? g.batch2 : 1;
  const int64_t b1 = g.batch / b2;
  CUtensorMap ta, tb;
  if (!make_map(&ta, A, ak, M, g.K, a_m, a_k, a_b ? b1 : 1, a_b, a_b2 ? b2 : 1, a_b2)) return false;
  if (!make_map(&tb, B, bk, N, g.K, b_n, b_k, b_b ? b1 : 1, b_b, b_b2 ? b2 : 1, b_b2)) return false;
  TcParams p{};
  p.M = M; p.N = N; p.K = g.K;
  p.batch = g.batch; p.batch2 = b2;
  p.a_kmajor = ak ? 1 : 0; p.b_kmajor = bk ? 1 : 0;
  p.a_b1 = a_b ? 1 : 0; p.a_b2 = a_b2 ? 1 : 0;
  p.b_b1 = b_b ? 1 : 0; p.b_b2 = b_b2 ? 1 : 0;
  p.C = g.C; p.c_m = c_m; p.c_n = c_n; p.c_batch = g.c_batch; p.c_batch2 = g.c_batch2;
  p.bias = g.bias; p.bias_m = swap ? 1 : 0; p.alpha = g.alpha; p.accumulate = g.accumulate;
  // 64-deep stages for a K-major B when every SM has many tiles to run
  const int64_t tiles_all = ((N + TC_BN - 1) / TC_BN) * ((M + TC_BM - 1) / TC_BM) * g.batch;
  const bool deep = bk && tiles_all >= 8 * device_sm_count() && g.K >= 512;
  p.sk = deep ? TcCfg<true, 2>::sk : TC_BK;
  const int64_t nk = (g.K + p.sk - 1) / p.sk;
  int splits = gemm_tc_splits(M, N, g.K, g.batch);
  if (splits > 1 && (!g.workspace || g.workspace_floats < (int64_t)splits * g.batch * M * N)) splits = 1;
  p.kps = (int)((nk + splits - 1) / splits);
  splits = (int)((nk + p.kps - 1) / p.kps);  // every split gets at least one K-stage
  p.splits = splits;
  p.ws = g.workspace;
  static const int trace = [] { const char* e = getenv("TG_GEMM_TRACE"); return e && e[0] == '1' ? 1 : 0; }();
  p.trace = trace;
  // rows of the kernel's tiles are the problem's m tiles, or its n tiles after a swap
  p.tri = splits == 1 ? (g.tri ? g.tri : g.tri_cols) : 0;
  p.tri_n = g.tri ? (swap ? 1 : 0) : (swap ? 0 : 1);
  // Output tensor map (row-major tiles {32 inner, 128 outer}); plain stores
  // when C's layout is not TMA-describable or the result accumulates.
  CUtensorMap tc;
  memset(&tc, 0, sizeof tc);
  static const bool tma_store_ok = [] { const char* e = getenv("TG_GEMM_TMA_STORE"); return !(e && e[0] == '0'); }();
  if (!tma_store_ok) {
    p.tma_store = 0;
  } else if (splits > 1) {
    p.tma_store = make_map(&tc, g.workspace, true, M, N, N, 1, (int64_t)splits * g.batch, M * N, 1, 0) ? 1 : 0;
  } else if (!g.accumulate && (c_n == 1 || c_m == 1)) {
    const bool cmaj = c_m == 1 && c_n != 1;
    const int64_t inner = cmaj ? M : N, outer = cmaj ? N : M, ld = cmaj ? c_n : c_m;
    p.tma_store = make_map(&tc, g.C, true, outer, inner, ld, 1, g.c_batch ? b1 : 1, g.c_batch,
                           g.c_batch2 ? b2 : 1, g.c_batch2) ? 1 : 0;
  }

  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(gemm_tc_kernel<true, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             TcCfg<true, 1>::smem) != cudaSuccess ||
        cudaFuncSetAttribute(gemm_tc_kernel<true, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             TcCfg<true, 2>::smem) != cudaSuccess ||
        cudaFuncSetAttribute(gemm_tc_kernel<false, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             TcCfg<false, 1>::smem) != cudaSuccess)
      return false;
    attr = true;
  }
  p.units = ((N + TC_BN - 1) / TC_BN) * ((M + TC_BM - 1) / TC_BM) * g.batch * splits;
  const int64_t sms = device_sm_count();
  const unsigned grid = (unsigned)(p.units < sms ? p.units : sms);
  if (deep) gemm_tc_kernel<true, 2><<<grid, 448, TcCfg<true, 2>::smem, s>>>(ta, tb, tc, p);
  else if (bk) gemm_tc_kernel<true, 1><<<grid, 448, TcCfg<true, 1>::smem, s>>>(ta, tb, tc, p);
  else gemm_tc_kernel<false, 1><<<grid, 448, TcCfg<false, 1>::smem, s>>>(ta, tb, tc, p);
  if (splits > 1) {
    int64_t total = g.batch * M * N;
    int64_t blocks = (total + 255) / 256, cap = (int64_t)device_sm_count() * 8;
    gemm_splitk_reduce<<<(unsigned)(blocks < cap ? blocks : cap), 256, 0, s>>>(p);
  }
  return true;
}

int gemm_tc_debug(int* out8) {
  return cudaMemcpyFromSymbol(out8, g_gemm_tc_dbg, 8 * sizeof(int)) == cudaSuccess ? 0 : 1;
}

int gemm_tc_trace(long long* out, int cap) {
  const int n = 12 * TC_TRACE_N;
  if (cap < n) return -1;
  return cudaMemcpyFromSymbol(out, g_gemm_tc_trace, n * sizeof(long long)) == cudaSuccess ? n : -1;
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
