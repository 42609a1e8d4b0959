// Causal attention forward on the 5th-generation tensor cores (head dim 64).
//
// Replaces, for one attention block, the reference's scores GEMM, scale,
// softmaxCausal and PV GEMM (src/codegen.ts:567-601, :656-689) when no
// dropout sits on the probabilities. It writes the same outputs as the
// warp-MMA forward kernel (kernels_attn.cu): O through its (merged-head)
// view and each query row's running max (in log2 units of the scaled score)
// and sum, which the backward kernels read.
//
// One CTA per (batch x head, 128-query block), key blocks of 128 up to the
// diagonal. 3xTF32 throughout, as in the GEMM: every f32 operand is split
// into hi (the raw bits; kind::tf32 truncates) and lo = x - hi, and each
// product is lo*hi + hi*lo + hi*hi.
//   S  = Q K^T   tcgen05.mma M=128 N=128, Q and K (hi and lo tiles) in shared
//                memory, S accumulated in TMEM columns [0, 128)
//   P  = exp2(S * scale * log2(e) - m)   row warps, one thread per query row
//                (its TMEM lane), online max and sum in registers; P's hi and
//                lo go to TMEM columns [192, 448) as the A operand of
//   PV = P V     tcgen05.mma M=128 N=64, V transposed in shared memory into
//                K-major hi and lo tiles; PV in TMEM columns [128, 192),
//                added by the row threads into O in registers (O * corr + PV,
//                f32 round-to-nearest).
// Warps 0-3 are the row warps (and split the tiles), warp 4 allocates TMEM
// and its lane 0 issues the TMA loads and the MMAs. Every wait is bounded; a
// timeout records a code in g_attn_tc_error and the CTA stops working but
// keeps its barriers.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>

#include "kernels.cuh"

namespace tg {

__device__ int g_attn_tc_error = 0;

namespace {

constexpr int AT_BQ = 128, AT_BK = 128, AT_D = 64;
constexpr int AT_SUB = 128 * 32 * 4;  // one 128-row x 32-float (128 B) swizzled sub-tile: 16 KB
constexpr long long AT_SPIN = 1ll << 22;
// shared memory (bytes from the 1 KB-aligned base)
constexpr int AT_Q = 0;                  // Q raw: 2 sub-tiles (head dims 0-31, 32-63)
constexpr int AT_QLO = AT_Q + 2 * AT_SUB;
constexpr int AT_K = AT_QLO + 2 * AT_SUB;
constexpr int AT_KLO = AT_K + 2 * AT_SUB;
constexpr int AT_V = AT_KLO + 2 * AT_SUB;  // V as landed: rows = keys
constexpr int AT_VT = AT_V + 2 * AT_SUB;   // V^T hi: 4 sub-tiles (32 keys each) of 64 rows x 128 B
constexpr int AT_VTLO = AT_VT + 4 * 8192;
constexpr int AT_END = AT_VTLO + 4 * 8192;
constexpr int AT_SMEM = AT_END + 1024 + 64;
// TMEM columns
constexpr uint32_t AT_TS = 0, AT_TPV = 128, AT_TPH = 192, AT_TPL = 320;

__device__ __forceinline__ uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void bar_init(uint64_t* b, uint32_t n) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(n));
}
__device__ __forceinline__ void bar_expect(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool bar_wait(uint64_t* b, uint32_t parity, int code) {
  for (long long i = 0; i < AT_SPIN; ++i) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok) : "r"(su32(b)), "r"(parity) : "memory");
    if (ok) return true;
  }
  atomicExch(&g_attn_tc_error, code);
  return false;
}
__device__ __forceinline__ void tma4(const CUtensorMap* tm, uint64_t* bar, void* dst, int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];"
      ::"r"(su32(dst)), "l"(tm), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(su32(bar))
      : "memory");
}
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) {  // K-major, 128B swizzle, 8-row groups 1 KB apart
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;                      // leading offset (unused for swizzled K-major)
  d |= (uint64_t)((1024 >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}
__device__ __forceinline__ void mma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n"
      ::"r"(d), "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n}\n"
      ::"r"(d), "r"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(bar)) : "memory");
}
__device__ __forceinline__ void tld32(uint32_t taddr, float (&r)[32]) {
  uint32_t u[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]), "=r"(u[6]), "=r"(u[7]),
        "=r"(u[8]), "=r"(u[9]), "=r"(u[10]), "=r"(u[11]), "=r"(u[12]), "=r"(u[13]), "=r"(u[14]), "=r"(u[15]),
        "=r"(u[16]), "=r"(u[17]), "=r"(u[18]), "=r"(u[19]), "=r"(u[20]), "=r"(u[21]), "=r"(u[22]), "=r"(u[23]),
        "=r"(u[24]), "=r"(u[25]), "=r"(u[26]), "=r"(u[27]), "=r"(u[28]), "=r"(u[29]), "=r"(u[30]), "=r"(u[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) r[i] = __uint_as_float(u[i]);
}
__device__ __forceinline__ void tst32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
      ::"r"(taddr), "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]),
        "f"(v[8]), "f"(v[9]), "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15]),
        "f"(v[16]), "f"(v[17]), "f"(v[18]), "f"(v[19]), "f"(v[20]), "f"(v[21]), "f"(v[22]), "f"(v[23]),
        "f"(v[24]), "f"(v[25]), "f"(v[26]), "f"(v[27]), "f"(v[28]), "f"(v[29]), "f"(v[30]), "f"(v[31])
      : "memory");
}
__device__ __forceinline__ float hi_of(float x) { return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); }

// lo = x - hi(x) of a swizzled K-major tile region (raw stays in place as hi).
__device__ __forceinline__ void lo_region(const uint8_t* raw, uint8_t* lo, int bytes, int t) {
  const float4* r4 = reinterpret_cast<const float4*>(raw);
  float4* l4 = reinterpret_cast<float4*>(lo);
  for (int q = t; q < bytes / 16; q += 128) {
    const float4 x = r4[q];
    l4[q] = make_float4(x.x - hi_of(x.x), x.y - hi_of(x.y), x.z - hi_of(x.z), x.w - hi_of(x.w));
  }
}

}  // namespace

__global__ void __launch_bounds__(160, 1) attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                                                             const __grid_constant__ CUtensorMap tmK,
                                                             const __grid_constant__ CUtensorMap tmV,
                                                             const __grid_constant__ AttnParams P) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024u - (su32(smem_raw) & 1023u)) & 1023u);
  uint64_t* tma_bar = reinterpret_cast<uint64_t*>(sm + AT_END);
  uint64_t* mma_bar = tma_bar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_bar + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, t = threadIdx.x;
  const bool issuer = threadIdx.x == 128;
  const int nqb = (P.T + AT_BQ - 1) / AT_BQ;
  const int qb = nqb - 1 - (int)blockIdx.x;  // longest rows first
  const int bh = blockIdx.y, b = bh / P.H, h = bh - b * P.H;
  const int q0 = qb * AT_BQ;

  if (threadIdx.x == 0) {
    bar_init(tma_bar, 1);
    bar_init(mma_bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 4) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(su32(tmem_slot)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  bool ok = true;
  uint32_t tph = 0, mph = 0;  // barrier phases

  // Q: both head-dim halves, then its lo part
  if (issuer) {
    bar_expect(tma_bar, 2 * AT_SUB);
    tma4(&tmQ, tma_bar, sm + AT_Q, 0, q0, h, b);
    tma4(&tmQ, tma_bar, sm + AT_Q + AT_SUB, 32, q0, h, b);
  }
  if (!bar_wait(tma_bar, tph, 1)) ok = false;
  ok = __all_sync(0xffffffffu, ok);  // warp-uniform, for the .sync.aligned TMEM accesses
  tph ^= 1u;
  if (t < 128 && ok) lo_region(sm + AT_Q, sm + AT_QLO, 2 * AT_SUB, t);

  const int r = (warp & 3) * 32 + lane;  // this row thread's query row / TMEM lane
  const int i = q0 + r;
  const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
  const float c2 = P.scale * 1.4426950408889634f;
  float m = -INFINITY, l = 0.f;
  float o[AT_D];
#pragma unroll
  for (int c = 0; c < AT_D; ++c) o[c] = 0.f;
  const uint32_t id_s = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(AT_BK >> 3) << 17) | ((uint32_t)(AT_BQ >> 4) << 24);
  const uint32_t id_pv = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(AT_D >> 3) << 17) | ((uint32_t)(AT_BQ >> 4) << 24);

  for (int kb = 0; kb <= qb; ++kb) {
    // a. K and V of this key block (issued during the previous block's
    //    softmax for every block after the first)
    auto load_kv = [&](int kbl) {
      bar_expect(tma_bar, 4 * AT_SUB);
      tma4(&tmK, tma_bar, sm + AT_K, 0, kbl * AT_BK, h, b);
      tma4(&tmK, tma_bar, sm + AT_K + AT_SUB, 32, kbl * AT_BK, h, b);
      tma4(&tmV, tma_bar, sm + AT_V, 0, kbl * AT_BK, h, b);
      tma4(&tmV, tma_bar, sm + AT_V + AT_SUB, 32, kbl * AT_BK, h, b);
    };
    if (issuer && ok && kb == 0) load_kv(0);
    if (ok && !bar_wait(tma_bar, tph, 2)) ok = false;
    ok = __all_sync(0xffffffffu, ok);
    tph ^= 1u;
    // b. K lo; V -> V^T hi and lo (row k = this thread's key)
    if (t < 128 && ok) {
      lo_region(sm + AT_K, sm + AT_KLO, 2 * AT_SUB, t);
      const int k = t;
      const uint8_t* vrow = sm + AT_V + k * 128;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          const float4 x = *reinterpret_cast<const float4*>(vrow + half * AT_SUB + ((ch ^ (k & 7)) << 4));
          const float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
          for (int w4 = 0; w4 < 4; ++w4) {
            const int n = half * 32 + ch * 4 + w4;  // head dim: row of V^T
            const uint32_t off = (uint32_t)(k >> 5) * 8192u + (uint32_t)n * 128u +
                                 (uint32_t)(((((k & 31) >> 2) ^ (n & 7))) << 4) + (uint32_t)((k & 3) << 2);
            *reinterpret_cast<float*>(sm + AT_VT + off) = xs[w4];
            *reinterpret_cast<float*>(sm + AT_VTLO + off) = xs[w4] - hi_of(xs[w4]);
          }
        }
      }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    asm volatile("bar.sync 1, 160;" ::: "memory");
    // c. S = Q K^T (previous PV reads of P and the previous S reads are done:
    //    the row threads passed the barrier after reading them)
    if (issuer && ok) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint64_t qh = sdesc(su32(sm + AT_Q)), ql = sdesc(su32(sm + AT_QLO));
      const uint64_t kh = sdesc(su32(sm + AT_K)), kl = sdesc(su32(sm + AT_KLO));
#pragma unroll
      for (int kk = 0; kk < AT_D / 8; ++kk) {
        const uint64_t o16 = (uint64_t)((kk >> 2) * (AT_SUB >> 4) + 2 * (kk & 3));
        mma_ss(tmem + AT_TS, ql + o16, kh + o16, id_s, kk ? 1u : 0u);
        mma_ss(tmem + AT_TS, qh + o16, kl + o16, id_s, 1u);
        mma_ss(tmem + AT_TS, qh + o16, kh + o16, id_s, 1u);
      }
      mma_commit(mma_bar);
    }
    if (ok && !bar_wait(mma_bar, mph, 3)) ok = false;
    ok = __all_sync(0xffffffffu, ok);
    mph ^= 1u;
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    // K and V of this block are consumed (V transposed, S computed): the
    // next block's loads run under this block's softmax and PV
    if (issuer && ok && kb < qb) load_kv(kb + 1);
    // d. online softmax of this row over the block; P hi and lo into TMEM
    float corr = 1.f;
    if (t < 128) {
      const bool edge = kb == qb || kb * AT_BK + AT_BK > P.T;
      float mx = -INFINITY;
      float sv[32];
      for (int c = 0; c < 4; ++c) {
        if (ok) tld32(tmem + lane_base + AT_TS + 32 * c, sv);
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int j = kb * AT_BK + 32 * c + e;
          const float x = (edge && (j > i || j >= P.T)) ? -INFINITY : sv[e] * c2;
          mx = fmaxf(mx, x);
        }
      }
      const float mn = fmaxf(m, mx);
      corr = exp2f(m - mn);
      m = mn;
      float sum = 0.f;
      for (int c = 0; c < 4; ++c) {
        if (ok) tld32(tmem + lane_base + AT_TS + 32 * c, sv);
        float ph[32], pl[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int j = kb * AT_BK + 32 * c + e;
          const float x = (edge && (j > i || j >= P.T)) ? -INFINITY : sv[e] * c2;
          const float p = exp2f(x - m);
          sum += p;
          ph[e] = p;
          pl[e] = p - hi_of(p);
        }
        if (ok) {
          tst32(tmem + lane_base + AT_TPH + 32 * c, ph);
          tst32(tmem + lane_base + AT_TPL + 32 * c, pl);
        }
      }
      l = l * corr + sum;
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    asm volatile("bar.sync 1, 160;" ::: "memory");
    // e. PV = P V
    if (issuer && ok) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint64_t vh = sdesc(su32(sm + AT_VT)), vl = sdesc(su32(sm + AT_VTLO));
#pragma unroll
      for (int kk = 0; kk < AT_BK / 8; ++kk) {
        const uint64_t o16 = (uint64_t)((kk >> 2) * (8192 >> 4) + 2 * (kk & 3));
        mma_ts(tmem + AT_TPV, tmem + AT_TPL + 8 * kk, vh + o16, id_pv, kk ? 1u : 0u);
        mma_ts(tmem + AT_TPV, tmem + AT_TPH + 8 * kk, vl + o16, id_pv, 1u);
        mma_ts(tmem + AT_TPV, tmem + AT_TPH + 8 * kk, vh + o16, id_pv, 1u);
      }
      mma_commit(mma_bar);
    }
    if (ok && !bar_wait(mma_bar, mph, 4)) ok = false;
    ok = __all_sync(0xffffffffu, ok);
    mph ^= 1u;
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    // f. O = O * corr + PV
    if (t < 128) {
      float pv[32];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        if (ok) tld32(tmem + lane_base + AT_TPV + 32 * c, pv);
        else
#pragma unroll
          for (int e = 0; e < 32; ++e) pv[e] = 0.f;
#pragma unroll
        for (int e = 0; e < 32; ++e) o[32 * c + e] = __fadd_rn(__fmul_rn(o[32 * c + e], corr), pv[e]);
      }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    asm volatile("bar.sync 1, 160;" ::: "memory");
  }
  if (t < 128 && ok && i < P.T) {
    const float inv = __frcp_rn(l);
    float* orow = P.o.p + (int64_t)b * P.o.s0 + (int64_t)h * P.o.s1 + (int64_t)i * P.o.s2;
#pragma unroll
    for (int c = 0; c < AT_D; ++c) orow[c * P.o.s3] = o[c] * inv;
    P.ml[2 * ((int64_t)bh * P.T + i)] = m;
    P.ml[2 * ((int64_t)bh * P.T + i) + 1] = l;
  }
  __syncthreads();
  if (warp == 4) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
  }
}

// ------------------------------------------------------------------- host --
static PFN_cuTensorMapEncodeTiled_v12000 at_encode() {
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

// {head dim, T, H, B} view with unit head-dim stride; boxes of 32 x 128 rows.
static bool at_map(CUtensorMap* tm, const AttnView& v, const AttnParams& P) {
  auto fn = at_encode();
  if (!fn || v.s3 != 1 || (reinterpret_cast<uintptr_t>(v.p) & 15)) return false;
  cuuint64_t dims[4] = {(cuuint64_t)P.D, (cuuint64_t)P.T, (cuuint64_t)P.H, (cuuint64_t)P.B};
  cuuint64_t strides[3] = {(cuuint64_t)(v.s2 * 4), (cuuint64_t)(v.s1 * 4), (cuuint64_t)(v.s0 * 4)};
  if (P.H == 1) strides[1] = 16;
  if (P.B == 1) strides[2] = 16;
  for (auto s : strides)
    if (s % 16 || s == 0) return false;
  cuuint32_t box[4] = {32, 128, 1, 1}, estr[4] = {1, 1, 1, 1};
  return fn(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, v.p, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

bool launch_attn_fwd_tc(const AttnParams& P, cudaStream_t s) {
  // opt-in (TG_ATTN_TC=1): measured slower than the warp-MMA forward so far
  const char* e = getenv("TG_ATTN_TC");
  if (!(e && e[0] == '1') || P.D != AT_D || P.dropout || P.T <= 0 || P.T > (1 << 24)) return false;
  CUtensorMap tq, tk, tv;
  if (!at_map(&tq, P.q, P) || !at_map(&tk, P.k, P) || !at_map(&tv, P.v, P)) return false;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(attn_fwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, AT_SMEM) != cudaSuccess)
      return false;
    attr = true;
  }
  dim3 grid((unsigned)((P.T + AT_BQ - 1) / AT_BQ), (unsigned)(P.B * P.H));
  attn_fwd_tc_kernel<<<grid, 160, AT_SMEM, s>>>(tq, tk, tv, P);
  return true;
}

int attn_tc_error_flag(bool reset) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_attn_tc_error, sizeof(int));
  if (reset) {
    int z = 0;
    cudaMemcpyToSymbol(g_attn_tc_error, &z, sizeof(int));
  }
  return v;
}

}  // namespace tg
