// Fused causal attention, forward and backward (flash-style, deterministic).
//
// Replaces the op chain the tracer emits for one attention block
// (src/ops.ts softmaxCausal/dropout; the kernels of src/codegen.ts:656-689
// and the matmul/permute kernels around them):
//
//   S  = (Q K^T) * scale            P  = softmaxCausal(S)      (row i keeps j <= i)
//   Pd = dropout(P)                 O  = Pd V
//
// and its gradient ops (dPd = dO V^T, dV = Pd^T dO, dP = dropout(dPd),
// dS = P * (dP - rowsum(dP * P)) * scale, dQ = dS K, dK = dS^T Q) without
// materialising S, P or Pd. The identity rowsum(dP * P) = rowsum(dO * O)
// (O = Pd V) gives the row term from O.
//
// Kernels (64 query or key rows per CTA, four warps of 16 rows):
//   attn_fwd   per (query block, head): key blocks up to the diagonal, online
//              softmax; writes O and each row's max m and sum l.
//   attn_rowdot  Dv[i] = dO_i . O_i
//   attn_bwd_kv  per (key block, head): query blocks from the diagonal on;
//              recomputes P = exp(S*scale - m) / l, accumulates dV and dK and
//              writes the lower-triangle blocks of dS.
//   attn_bwd_q   per (query block, head): dQ = dS K over key blocks up to the
//              diagonal.
// Every sum is a fixed sequence per thread: results do not depend on
// scheduling. Contractions use mma.sync m16n8k8 TF32 with operands split
// hi + lo (3 products: lo*hi + hi*lo + hi*hi), f32 accumulation.
// Loops over the contraction dimension that read only shared memory stay
// rolled (`unroll 1`): fully unrolled, the kernels outgrew the instruction
// cache (the top stall was "no instruction") and ran about 17% slower.
// Dropout masks hash the flat [B, H, T, T] element index exactly as the
// elementwise dropout kernels do, so fused and unfused runs drop the same
// elements.
#include "kernels.cuh"

namespace tg {

namespace {

constexpr int AB = 64;      // rows per tile
constexpr int SPP = AB + 4; // staging row stride (floats)

__device__ __forceinline__ uint32_t attn_hash(uint32_t h) {
  h = h * 747796405u + 2891336453u;
  h = ((h >> ((h >> 28u) + 4u)) ^ h) * 277803737u;
  return (h >> 22u) ^ h;
}

__device__ __forceinline__ void split_tf32(float x, uint32_t& hi, uint32_t& lo) {
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(hi) : "f"(x));
  lo = __float_as_uint(x - __uint_as_float(hi));
}

__device__ __forceinline__ void mma8(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                     uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// An A fragment (rows g, g+8; columns t, t+4) split into TF32 hi and lo.
struct AFrag { uint32_t h[4], l[4]; };
__device__ __forceinline__ AFrag afrag(float a0, float a1, float a2, float a3) {
  AFrag f;
  split_tf32(a0, f.h[0], f.l[0]);
  split_tf32(a1, f.h[1], f.l[1]);
  split_tf32(a2, f.h[2], f.l[2]);
  split_tf32(a3, f.h[3], f.l[3]);
  return f;
}
// A fragment of rows r, r+8 at column c of a row-major shared tile.
__device__ __forceinline__ AFrag afrag_at(const float* row_g, int stride) {
  return afrag(row_g[0], row_g[8 * stride], row_g[4], row_g[8 * stride + 4]);
}

// c[n] += a * b_n for N independent 16x8x8 steps (n = N0 .. N0 + N - 1),
// issued as three passes over n (lo*hi, then hi*lo, then hi*hi) so that
// consecutive MMAs never wait on one accumulator. Both operands are split
// (3xTF32); the dropped lo*lo term is about 2^-22 relative. ldb(n, b0, b1)
// fetches the two B values of step n.
template <int N0, int N, int C, class LoadB>
__device__ __forceinline__ void mma3n(float (&c)[C][4], const AFrag& a, LoadB ldb) {
  uint32_t bh[N][2], bl[N][2];
#pragma unroll
  for (int n = 0; n < N; ++n) {
    float b0, b1;
    ldb(N0 + n, b0, b1);
    split_tf32(b0, bh[n][0], bl[n][0]);
    split_tf32(b1, bh[n][1], bl[n][1]);
  }
#pragma unroll
  for (int n = 0; n < N; ++n) mma8(c[N0 + n], a.l[0], a.l[1], a.l[2], a.l[3], bh[n][0], bh[n][1]);
#pragma unroll
  for (int n = 0; n < N; ++n) mma8(c[N0 + n], a.h[0], a.h[1], a.h[2], a.h[3], bl[n][0], bl[n][1]);
#pragma unroll
  for (int n = 0; n < N; ++n) mma8(c[N0 + n], a.h[0], a.h[1], a.h[2], a.h[3], bh[n][0], bh[n][1]);
}

__device__ __forceinline__ float vld(const AttnView& v, int b, int h, int t, int c) {
  return v.p[(int64_t)b * v.s0 + (int64_t)h * v.s1 + (int64_t)t * v.s2 + (int64_t)c * v.s3];
}
__device__ __forceinline__ void vst(const AttnView& v, int b, int h, int t, int c, float x) {
  v.p[(int64_t)b * v.s0 + (int64_t)h * v.s1 + (int64_t)t * v.s2 + (int64_t)c * v.s3] = x;
}

__device__ __forceinline__ uint32_t smem_u32a(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// Rows [r0, r0 + 64), columns [0, D) of a (b, h) slice into shared memory
// (row stride S); zeros past row T and past column ncol, which are never
// read. Unit-stride 16-byte aligned rows go by cp.async (all of a thread's
// chunks in flight at once; the caller waits with cp_wait); other views by
// plain loads.
template <int D, int S>
__device__ __forceinline__ void load_tile(float* dst, const AttnView& v, int b, int h, int r0, int T,
                                          int ncol = D) {
  const bool vec = v.s3 == 1 && ((v.s0 | v.s1 | v.s2) & 3) == 0 && (ncol & 3) == 0 &&
                   !(reinterpret_cast<uintptr_t>(v.p) & 15);
  if (vec) {
    constexpr int CPR = D / 4;
    const float* base = v.p + (int64_t)b * v.s0 + (int64_t)h * v.s1;
    for (int e = threadIdx.x; e < AB * CPR; e += blockDim.x) {
      const int r = e / CPR, c = (e - r * CPR) * 4;
      const int t = r0 + r;
      const bool in = t < T && c < ncol;
      const float* src = in ? base + (int64_t)t * v.s2 + c : v.p;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32a(dst + r * S + c)), "l"(src),
                   "r"(in ? 16 : 0)
                   : "memory");
    }
  } else {
    for (int e = threadIdx.x; e < AB * D; e += blockDim.x) {
      const int r = e / D, c = e - r * D;
      dst[r * S + c] = (r0 + r < T && c < ncol) ? vld(v, b, h, r0 + r, c) : 0.f;
    }
  }
}
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Dropout factor of the element whose flat [B, H, T, T] index plus the
// rank's offset is `idx` (only its low 32 bits enter the hash, so callers
// form it in 32-bit arithmetic).
__device__ __forceinline__ float drop_factor(const AttnParams& P, uint32_t seed, uint32_t idx) {
  if (!P.dropout) return 1.f;
  const uint32_t hsh = attn_hash(seed ^ P.salt ^ idx);
  return __uint2float_rn(hsh) * 2.3283064365386963e-10f >= P.p ? P.keep_scale : 0.f;
}
// Low 32 bits of the flat index of element (i, 0) of head bh, with the offset.
__device__ __forceinline__ uint32_t drop_row(const AttnParams& P, int bh, int i) {
  return (uint32_t)(P.drop_off + ((int64_t)bh * P.T + i) * P.T);
}
// exp(x * scale - m) is evaluated as exp2(x * c - m2), c = scale * log2(e):
// the forward keeps the running max m2 in these units and the backward
// recomputes the probabilities the same way.
constexpr float LOG2E = 1.4426950408889634f;

}  // namespace

// ------------------------------------------------------------------ forward --
template <int D>
__global__ void __launch_bounds__(128) attn_fwd_kernel(const __grid_constant__ AttnParams P) {
  constexpr int SQ = D + 4, SV = D + 8;
  extern __shared__ float sm[];
  float* sQ = sm;
  float* sK = sQ + AB * SQ;
  float* sV = sK + AB * SQ;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  float* sP = sV + AB * SV + w * 16 * SPP;
  const int nqb = (P.T + AB - 1) / AB;
  const int qb = nqb - 1 - (int)blockIdx.x;  // longest rows first
  const int bh = blockIdx.y, b = bh / P.H, h = bh - b * P.H;
  const int q0 = qb * AB;
  const uint32_t seed = P.seed ? (uint32_t)(*P.seed) : 0u;

  load_tile<D, SQ>(sQ, P.q, b, h, q0, P.T);
  cp_wait();
  __syncthreads();
  AFrag qa[D / 8];
#pragma unroll
  for (int kk = 0; kk < D / 8; ++kk) qa[kk] = afrag_at(sQ + (16 * w + g) * SQ + 8 * kk + t, SQ);
  const int i0 = q0 + 16 * w + g, i1 = i0 + 8;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  float oacc[D / 8][4];
#pragma unroll
  for (int n = 0; n < D / 8; ++n) oacc[n][0] = oacc[n][1] = oacc[n][2] = oacc[n][3] = 0.f;
  const float c2 = P.scale * LOG2E;

  for (int kb = 0; kb <= qb; ++kb) {
    __syncthreads();
    load_tile<D, SQ>(sK, P.k, b, h, kb * AB, P.T);
    load_tile<D, SV>(sV, P.v, b, h, kb * AB, P.T);
    cp_wait();
    __syncthreads();
    float s[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 8; ++kk) {
      const float* kb8 = sK + g * SQ + 8 * kk + t;
      const auto ldk = [&](int nt, float& b0, float& b1) { b0 = kb8[8 * nt * SQ]; b1 = kb8[8 * nt * SQ + 4]; };
      mma3n<0, 4>(s, qa[kk], ldk);
      mma3n<4, 4>(s, qa[kk], ldk);
    }
    // scale (in log2 units), causal/tail mask, online softmax over this key block
    const bool edge = kb == qb || kb * AB + AB > P.T;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float x = s[nt][e] * c2;
        if (edge) {
          const int j = kb * AB + 8 * nt + 2 * t + (e & 1), i = e < 2 ? i0 : i1;
          if (j > i || j >= P.T) x = -INFINITY;
        }
        s[nt][e] = x;
        mx[e >> 1] = fmaxf(mx[e >> 1], x);
      }
    float alpha[2], sum[2] = {0.f, 0.f};
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      const float mn = fmaxf(mrow[r], mx[r]);
      alpha[r] = exp2f(mrow[r] - mn);
      mrow[r] = mn;
    }
    const uint32_t dr0 = drop_row(P, bh, i0) + (uint32_t)(kb * AB), dr1 = drop_row(P, bh, i1) + (uint32_t)(kb * AB);
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = e >> 1, jl = 8 * nt + 2 * t + (e & 1);
        const float pe = exp2f(s[nt][e] - mrow[r]);
        sum[r] += pe;
        sP[(g + 8 * r) * SPP + jl] = pe * drop_factor(P, seed, (r ? dr1 : dr0) + (uint32_t)jl);
      }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      sum[r] += __shfl_xor_sync(0xffffffffu, sum[r], 1);
      sum[r] += __shfl_xor_sync(0xffffffffu, sum[r], 2);
      lrow[r] = lrow[r] * alpha[r] + sum[r];
    }
#pragma unroll
    for (int n = 0; n < D / 8; ++n) {
      oacc[n][0] *= alpha[0]; oacc[n][1] *= alpha[0];
      oacc[n][2] *= alpha[1]; oacc[n][3] *= alpha[1];
    }
    __syncwarp();
    // O += Pd V
#pragma unroll 1
    for (int kk = 0; kk < 8; ++kk) {
      const AFrag pa = afrag_at(sP + g * SPP + 8 * kk + t, SPP);
      const float* vr = sV + (8 * kk + t) * SV + g;
      mma3n<0, D / 8>(oacc, pa, [&](int n, float& b0, float& b1) { b0 = vr[8 * n]; b1 = vr[8 * n + 4 * SV]; });
    }
    __syncwarp();
  }
  const float inv_l[2] = {__frcp_rn(lrow[0]), __frcp_rn(lrow[1])};
#pragma unroll
  for (int n = 0; n < D / 8; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int r = e >> 1, i = r ? i1 : i0;
      if (i < P.T) vst(P.o, b, h, i, 8 * n + 2 * t + (e & 1), oacc[n][e] * inv_l[r]);
    }
  if (t == 0) {
    if (i0 < P.T) { P.ml[2 * ((int64_t)bh * P.T + i0)] = mrow[0]; P.ml[2 * ((int64_t)bh * P.T + i0) + 1] = lrow[0]; }
    if (i1 < P.T) { P.ml[2 * ((int64_t)bh * P.T + i1)] = mrow[1]; P.ml[2 * ((int64_t)bh * P.T + i1) + 1] = lrow[1]; }
  }
}

// Dv[bh, i] = sum_c dO(b, h, i, c) * O(b, h, i, c): one warp per row.
template <int D>
__global__ void __launch_bounds__(256) attn_rowdot_kernel(const __grid_constant__ AttnParams P) {
  const int64_t rows = (int64_t)P.B * P.H * P.T;
  const int lane = threadIdx.x & 31;
  for (int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows;
       r += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int i = (int)(r % P.T);
    const int bh = (int)(r / P.T), b = bh / P.H, h = bh - b * P.H;
    float acc = 0.f;
    for (int c = lane; c < D; c += 32) acc += vld(P.dout, b, h, i, c) * vld(P.o, b, h, i, c);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) P.dv_row[r] = acc;
  }
}

// ------------------------------------------------------- backward: dK, dV --
template <int D>
__global__ void __launch_bounds__(128, 3) attn_bwd_kv_kernel(const __grid_constant__ AttnParams P) {
  constexpr int SQ = D + 4;
  extern __shared__ float sm[];
  float* sK = sm;
  float* sV = sK + AB * SQ;
  float* sQ = sV + AB * SQ;
  float* sO = sQ + AB * SQ;  // dO
  float* sML = sO + AB * SQ;   // [64][2]
  float* sDv = sML + 2 * AB;   // [64]
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  float* sP = sDv + AB + w * 16 * SPP;
  const int nb = (P.T + AB - 1) / AB;
  const int kb = (int)blockIdx.x;  // key blocks near the start see the most query blocks
  const int bh = blockIdx.y, b = bh / P.H, h = bh - b * P.H;
  const uint32_t seed = P.seed ? (uint32_t)(*P.seed) : 0u;

  load_tile<D, SQ>(sK, P.k, b, h, kb * AB, P.T);
  load_tile<D, SQ>(sV, P.v, b, h, kb * AB, P.T);
  const int j0 = kb * AB + 16 * w + g, j1 = j0 + 8;  // this thread's key rows
  float dk[D / 8][4], dv[D / 8][4];
#pragma unroll
  for (int n = 0; n < D / 8; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk[n][e] = dv[n][e] = 0.f;

  for (int qb = kb; qb < nb; ++qb) {
    __syncthreads();
    load_tile<D, SQ>(sQ, P.q, b, h, qb * AB, P.T);
    load_tile<D, SQ>(sO, P.dout, b, h, qb * AB, P.T);
    for (int r = threadIdx.x; r < AB; r += blockDim.x) {
      const int i = qb * AB + r;
      const int64_t ri = (int64_t)bh * P.T + i;
      sML[2 * r] = i < P.T ? P.ml[2 * ri] : 0.f;
      sML[2 * r + 1] = i < P.T ? __frcp_rn(P.ml[2 * ri + 1]) : 0.f;  // 1 / l
      sDv[r] = i < P.T ? P.dv_row[ri] : 0.f;
    }
    cp_wait();
    __syncthreads();
    // S^T (16 keys x 64 queries) = K_w Q^T and dPd^T = V_w dO^T
    float st[8][4], dp[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      st[nt][0] = st[nt][1] = st[nt][2] = st[nt][3] = 0.f;
      dp[nt][0] = dp[nt][1] = dp[nt][2] = dp[nt][3] = 0.f;
    }
#pragma unroll 1
    for (int kk = 0; kk < D / 8; ++kk) {
      const AFrag ka = afrag_at(sK + (16 * w + g) * SQ + 8 * kk + t, SQ);
      const AFrag va = afrag_at(sV + (16 * w + g) * SQ + 8 * kk + t, SQ);
      const float* qr = sQ + g * SQ + 8 * kk + t;
      const float* orr = sO + g * SQ + 8 * kk + t;
      const auto ldq = [&](int nt, float& b0, float& b1) { b0 = qr[8 * nt * SQ]; b1 = qr[8 * nt * SQ + 4]; };
      const auto ldo = [&](int nt, float& b0, float& b1) { b0 = orr[8 * nt * SQ]; b1 = orr[8 * nt * SQ + 4]; };
      mma3n<0, 4>(st, ka, ldq);
      mma3n<0, 4>(dp, va, ldo);
      mma3n<4, 4>(st, ka, ldq);
      mma3n<4, 4>(dp, va, ldo);
    }
    // P^T, dropout, dS^T; Pd^T staged for dV
    const float c2 = P.scale * LOG2E;
    const bool edge = qb == kb || qb * AB + AB > P.T || kb * AB + AB > P.T;
    // flat index of (i, j) = (bh*T + i)*T + j: the key row's base plus i*T
    const uint32_t db0 = (uint32_t)(P.drop_off + (int64_t)bh * P.T * P.T + j0) + (uint32_t)(qb * AB) * (uint32_t)P.T;
    const uint32_t db1 = db0 + 8u;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = e >> 1, ql = 8 * nt + 2 * t + (e & 1);
        bool ok = true;
        if (edge) {
          const int i = qb * AB + ql, j = r ? j1 : j0;
          ok = j <= i && i < P.T && j < P.T;
        }
        const float p = ok ? exp2f(st[nt][e] * c2 - sML[2 * ql]) * sML[2 * ql + 1] : 0.f;
        const float f = ok ? drop_factor(P, seed, (r ? db1 : db0) + (uint32_t)ql * (uint32_t)P.T) : 0.f;
        sP[(g + 8 * r) * SPP + ql] = __fmul_rn(p, f);
        const float dpe = __fmul_rn(dp[nt][e], f);
        st[nt][e] = __fmul_rn(__fmul_rn(__fsub_rn(dpe, sDv[ql]), p), P.scale);  // dS^T
      }
    __syncwarp();
    // dV += Pd^T dO
#pragma unroll 1
    for (int kk = 0; kk < 8; ++kk) {
      const AFrag pa = afrag_at(sP + g * SPP + 8 * kk + t, SPP);
      const float* orr = sO + (8 * kk + t) * SQ + g;
      mma3n<0, D / 8>(dv, pa, [&](int n, float& b0, float& b1) { b0 = orr[8 * n]; b1 = orr[8 * n + 4 * SQ]; });
    }
    __syncwarp();
    // dS: staged for dK and written out (queries of this block, this warp's keys)
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = e >> 1, ql = 8 * nt + 2 * t + (e & 1);
        sP[(g + 8 * r) * SPP + ql] = st[nt][e];
        const int i = qb * AB + ql, j = r ? j1 : j0;
        if (i < P.T && j < P.T) P.ds[((int64_t)bh * P.T + i) * P.ds_ld + j] = st[nt][e];
      }
    __syncwarp();
    // dK += dS^T Q
#pragma unroll 1
    for (int kk = 0; kk < 8; ++kk) {
      const AFrag pa = afrag_at(sP + g * SPP + 8 * kk + t, SPP);
      const float* qr = sQ + (8 * kk + t) * SQ + g;
      mma3n<0, D / 8>(dk, pa, [&](int n, float& b0, float& b1) { b0 = qr[8 * n]; b1 = qr[8 * n + 4 * SQ]; });
    }
  }
#pragma unroll
  for (int n = 0; n < D / 8; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int j = (e >> 1) ? j1 : j0, c = 8 * n + 2 * t + (e & 1);
      if (j < P.T) {
        vst(P.dk, b, h, j, c, dk[n][e]);
        vst(P.dv, b, h, j, c, dv[n][e]);
      }
    }
}

// ------------------------------------------------------------ backward: dQ --
template <int D>
__global__ void __launch_bounds__(128) attn_bwd_q_kernel(const __grid_constant__ AttnParams P) {
  constexpr int SK = D + 8;
  extern __shared__ float sm[];
  float* sS = sm;              // dS block [64][SPP]
  float* sK = sS + AB * SPP;   // K block [64][SK]
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int nqb = (P.T + AB - 1) / AB;
  const int qb = nqb - 1 - (int)blockIdx.x;
  const int bh = blockIdx.y, b = bh / P.H, h = bh - b * P.H;
  const int i0 = qb * AB + 16 * w + g, i1 = i0 + 8;
  float dq[D / 8][4];
#pragma unroll
  for (int n = 0; n < D / 8; ++n) dq[n][0] = dq[n][1] = dq[n][2] = dq[n][3] = 0.f;
  for (int kb = 0; kb <= qb; ++kb) {
    __syncthreads();
    // rows of dS; the backward key-block kernel wrote every entry of the
    // blocks on or below the diagonal (zeros above it within the diagonal block)
    const AttnView dsv{P.ds, 0, P.T * P.ds_ld, P.ds_ld, 1};
    load_tile<AB, SPP>(sS, AttnView{dsv.p + (int64_t)kb * AB, 0, dsv.s1, dsv.s2, 1}, 0, bh, qb * AB, P.T,
                       min(AB, P.T - kb * AB));
    load_tile<D, SK>(sK, P.k, b, h, kb * AB, P.T);
    cp_wait();
    __syncthreads();
#pragma unroll 1
    for (int kk = 0; kk < 8; ++kk) {
      const AFrag sa = afrag_at(sS + (16 * w + g) * SPP + 8 * kk + t, SPP);
      const float* kr = sK + (8 * kk + t) * SK + g;
      mma3n<0, D / 8>(dq, sa, [&](int n, float& b0, float& b1) { b0 = kr[8 * n]; b1 = kr[8 * n + 4 * SK]; });
    }
  }
#pragma unroll
  for (int n = 0; n < D / 8; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int i = (e >> 1) ? i1 : i0;
      if (i < P.T) vst(P.dq, b, h, i, 8 * n + 2 * t + (e & 1), dq[n][e]);
    }
}

// ---------------------------------------------------------------- host --
template <int D>
static void set_smem(const void* fn, int bytes) {
  cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

template <int D>
static void attn_fwd_t(const AttnParams& P, cudaStream_t s) {
  const int smem = (AB * (D + 4) * 2 + AB * (D + 8) + 4 * 16 * SPP) * 4;
  static bool init = false;
  if (!init) { set_smem<D>((const void*)attn_fwd_kernel<D>, smem); init = true; }
  const dim3 grid((P.T + AB - 1) / AB, P.B * P.H);
  attn_fwd_kernel<D><<<grid, 128, smem, s>>>(P);
}

template <int D>
static void attn_bwd_t(const AttnParams& P, cudaStream_t s) {
  const int nb = (P.T + AB - 1) / AB;
  const int64_t rows = (int64_t)P.B * P.H * P.T;
  const int64_t rb = (rows * 32 + 255) / 256, cap = (int64_t)device_sm_count() * 16;
  attn_rowdot_kernel<D><<<(unsigned)(rb < cap ? rb : cap), 256, 0, s>>>(P);
  const int smem_kv = (AB * (D + 4) * 4 + 3 * AB + 4 * 16 * SPP) * 4;
  const int smem_q = (AB * SPP + AB * (D + 8)) * 4;
  static bool init = false;
  if (!init) {
    set_smem<D>((const void*)attn_bwd_kv_kernel<D>, smem_kv);
    set_smem<D>((const void*)attn_bwd_q_kernel<D>, smem_q);
    init = true;
  }
  attn_bwd_kv_kernel<D><<<dim3(nb, P.B * P.H), 128, smem_kv, s>>>(P);
  attn_bwd_q_kernel<D><<<dim3(nb, P.B * P.H), 128, smem_q, s>>>(P);
}

bool attn_supported_dim(int d) { return d == 16 || d == 32 || d == 64; }

void launch_attn_fwd(const AttnParams& P, cudaStream_t s) {
  if (launch_attn_fwd_tc(P, s)) return;
  if (P.D == 64) attn_fwd_t<64>(P, s);
  else if (P.D == 32) attn_fwd_t<32>(P, s);
  else attn_fwd_t<16>(P, s);
}

void launch_attn_bwd(const AttnParams& P, cudaStream_t s) {
  if (P.D == 64) attn_bwd_t<64>(P, s);
  else if (P.D == 32) attn_bwd_t<32>(P, s);
  else attn_bwd_t<16>(P, s);
}

}  // namespace tg
