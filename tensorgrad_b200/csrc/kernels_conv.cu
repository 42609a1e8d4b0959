// conv2d and its two gradients as GEMMs (NCHW, groups, stride, zero padding).
//
// The reference emits one direct WGSL kernel per conv op (src/codegen.ts:916-1093);
// its CPU evaluator defines the sums (test/_eval.ts conv2d cases). Here each op
// becomes a column gather plus a contraction on the GEMM path (tcgen05 3xTF32
// where the operands are TMA-describable, the SIMT kernel otherwise):
//
//   col[k, b*HWo + p]  = x[b, g*cpg + cl, ho*sH + kh - pH, wo*sW + kw - pW]   (0 outside)
//                        k = (cl*kH + kh)*kW + kw,  p = ho*Wout + wo
//   forward      y[b, g*opg + o, p]  = sum_k W_g[o, k] * col[k, b*HWo + p]        (batched over b)
//   input grad   dcol[k, b*HWo + p]  = sum_o W_g[o, k] * dy[b, g*opg + o, p]      (batched over b)
//                dx[b, ci, h, w]     = sum over (kh, kw) hitting (h, w) of dcol     (gather, no atomics)
//   weight grad  dW_g[o, k]          = sum_{b,p} dyT[g*opg + o, b*HWo + p] * col[k, b*HWo + p]
//                                      (one long-K contraction, split-K on the GEMM path)
//
// col is [Kg, B*HWo] so every contraction reads it with unit stride along
// b*HWo; dyT is dy with its batch and channel axes swapped. All three use
// op-local scratch: [col | dyT | GEMM workspace].
#include <cstdio>
#include "kernels.cuh"

namespace tg {

// One (k, b) row of col per block iteration: the tap and sample are decoded
// once per row. VEC: each thread writes four consecutive outputs with one
// float4 store (HWo % 4 == 0), issuing its four gathered loads together.
template <bool VEC>
__global__ void __launch_bounds__(256) im2col_kernel(const __grid_constant__ ConvDesc c, int g,
                                                     const float* __restrict__ x, float* __restrict__ col) {
  const int cpg = c.Cin / c.G, kk = c.kH * c.kW, hwo = c.Hout * c.Wout;
  const int64_t bhw = (int64_t)c.B * hwo;
  const int rows = cpg * kk * c.B;
  for (int row = blockIdx.x; row < rows; row += gridDim.x) {
    const int k = row / c.B, b = row - k * c.B;
    const int cl = k / kk, kr = k - cl * kk;
    const int kh = kr / c.kW, kw = kr - kh * c.kW;
    const float* xp = x + ((int64_t)b * c.Cin + g * cpg + cl) * c.H * c.W;
    float* out = col + (int64_t)k * bhw + (int64_t)b * hwo;
    if (VEC) {
      for (int p = 4 * threadIdx.x; p < hwo; p += 4 * blockDim.x) {
        int ho = p / c.Wout, wo = p - ho * c.Wout;
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int hi = ho * c.sH + kh - c.pH, wi = wo * c.sW + kw - c.pW;
          v[j] = (hi >= 0 && hi < c.H && wi >= 0 && wi < c.W) ? __ldg(xp + hi * c.W + wi) : 0.f;
          if (++wo == c.Wout) { wo = 0; ++ho; }
        }
        *reinterpret_cast<float4*>(out + p) = make_float4(v[0], v[1], v[2], v[3]);
      }
    } else {
      for (int p = threadIdx.x; p < hwo; p += blockDim.x) {
        const int ho = p / c.Wout, wo = p - ho * c.Wout;
        const int hi = ho * c.sH + kh - c.pH, wi = wo * c.sW + kw - c.pW;
        out[p] = (hi >= 0 && hi < c.H && wi >= 0 && wi < c.W) ? xp[hi * c.W + wi] : 0.f;
      }
    }
  }
}

// dx[b, g*cpg + cl, h, w] = sum of dcol over the (kh, kw) taps whose output
// position lands on (h, w); taps in ascending (kh, kw) order. One (b, cl)
// plane per block iteration. KH/KW > 0 fix the window at compile time so
// every tap's load is issued unconditionally-addressed and predicated.
template <int KH, int KW>
__global__ void __launch_bounds__(256) col2im_kernel(const __grid_constant__ ConvDesc c, int g,
                                                     const float* __restrict__ dcol, float* __restrict__ dx) {
  const int kH = KH > 0 ? KH : c.kH, kW = KW > 0 ? KW : c.kW;
  const int cpg = c.Cin / c.G, kk = kH * kW, hwo = c.Hout * c.Wout, hw = c.H * c.W;
  const int64_t bhw = (int64_t)c.B * hwo;
  const int planes = c.B * cpg;
  for (int pl = blockIdx.x; pl < planes; pl += gridDim.x) {
    const int b = pl / cpg, cl = pl - b * cpg;
    const float* src = dcol + (int64_t)cl * kk * bhw + (int64_t)b * hwo;
    float* dst = dx + ((int64_t)b * c.Cin + g * cpg + cl) * hw;
    for (int r = threadIdx.x; r < hw; r += blockDim.x) {
      const int hi = r / c.W, wi = r - hi * c.W;
      float s = 0.f;
#pragma unroll
      for (int kh = 0; kh < kH; ++kh) {
        const int nh = hi + c.pH - kh;
        const int ho = nh / c.sH;
        const bool okh = nh >= 0 && nh - ho * c.sH == 0 && ho < c.Hout;
#pragma unroll
        for (int kw = 0; kw < kW; ++kw) {
          const int nw = wi + c.pW - kw;
          const int wo = nw / c.sW;
          const bool ok = okh && nw >= 0 && nw - wo * c.sW == 0 && wo < c.Wout;
          const float v = ok ? __ldg(src + (int64_t)(kh * kW + kw) * bhw + ho * c.Wout + wo) : 0.f;
          s += v;
        }
      }
      dst[r] = s;
    }
  }
}

// dyT[ch, b*hw + p] = dy[b, ch, p]: one (b, ch) run of hw floats per block
// iteration, moved whole.
__global__ void __launch_bounds__(256) swap_bc_kernel(const float* __restrict__ dy, float* __restrict__ dyt,
                                                      int B, int C, int hw) {
  const int rows = B * C;
  for (int row = blockIdx.x; row < rows; row += gridDim.x) {
    const int b = row / C, ch = row - b * C;
    const float* src = dy + (int64_t)row * hw;
    float* dst = dyt + ((int64_t)ch * B + b) * hw;
    for (int p = threadIdx.x; p < hw; p += blockDim.x) dst[p] = src[p];
  }
}

static unsigned row_grid(int64_t rows) {
  int64_t cap = (int64_t)device_sm_count() * 8;
  return (unsigned)(rows < cap ? (rows < 1 ? 1 : rows) : cap);
}

static void launch_im2col(const ConvDesc& c, int g, const float* x, float* col, cudaStream_t s) {
  const int64_t rows = (int64_t)(c.Cin / c.G) * c.kH * c.kW * c.B;
  // block width follows the row (one float4 per thread) so short rows do
  // not leave most lanes idle; more resident blocks keep more loads in flight
  const int hwo = c.Hout * c.Wout;
  if (hwo % 4 == 0 && !(reinterpret_cast<uintptr_t>(col) & 15)) {
    int t = ((hwo / 4 + 31) / 32) * 32;
    t = t < 256 ? t : 256;
    const int64_t cap = (int64_t)device_sm_count() * (2048 / t);
    im2col_kernel<true><<<(unsigned)(rows < cap ? rows : cap), t, 0, s>>>(c, g, x, col);
  } else {
    im2col_kernel<false><<<row_grid(rows), 256, 0, s>>>(c, g, x, col);
  }
}

static int64_t align64(int64_t n) { return (n + 63) & ~int64_t(63); }

static void gemm(const GemmDesc& g, cudaStream_t s) {
  if (!launch_gemm_tc(g, s)) launch_gemm_simt(g, s);
}

static GemmDesc base_desc(float* ws, int64_t ws_floats) {
  GemmDesc g{};
  g.alpha = 1.f;
  g.batch = 1;
  g.batch2 = 1;
  g.ldc_n = 1;
  g.workspace = ws;
  g.workspace_floats = ws_floats;
  return g;
}

// Workspace the GEMM path may use for split-K (tensor-core or SIMT) on an
// M x N x K problem with `batch` output tiles; SIMT splits are capped by what
// it is given, so the tensor-core figure plus one full output covers both.
static int64_t gemm_ws(int64_t M, int64_t N, int64_t K, int64_t batch) {
  return gemm_tc_workspace_floats(M, N, K, batch) + gemm_tc_workspace_floats(N, M, K, batch);
}

int64_t conv_gemm_scratch_floats(const ConvDesc& c, int which) {
  const int cpg = c.Cin / c.G, opg = c.Cout / c.G;
  const int64_t kg = (int64_t)cpg * c.kH * c.kW, hwo = (int64_t)c.Hout * c.Wout, bhw = c.B * hwo;
  const int64_t col = align64(kg * bhw);
  if (which == 0) return col + align64(gemm_ws(opg, hwo, kg, c.B));
  if (which == 1) return col + align64(gemm_ws(kg, hwo, opg, c.B));
  int64_t ws = gemm_ws(opg, kg, bhw, 1);
  ws = ws > opg * kg * 32 ? ws : opg * kg * 32;  // room for the SIMT kernel's own K-splits
  return col + align64((int64_t)c.Cout * bhw) + align64(ws);
}

static std::string gemm_label(const char* kind, const GemmDesc& d) {
  char b[128];
  snprintf(b, sizeof b, "%s|M=%lld N=%lld K=%lld b=%lld", kind, (long long)d.M, (long long)d.N, (long long)d.K,
           (long long)d.batch);
  return b;
}

void emit_conv(int which, const ConvDesc& c, const float* in0, const float* in1, float* out, float* scratch,
               int64_t scratch_floats, const ConvEmit& add) {
  const int cpg = c.Cin / c.G, opg = c.Cout / c.G;
  const int64_t kg = (int64_t)cpg * c.kH * c.kW, hwo = (int64_t)c.Hout * c.Wout, bhw = c.B * hwo;
  float* col = scratch;
  if (which == 0) {  // in0 = x, in1 = w, out = y
    const float *x = in0, *w = in1;
    float* ws = scratch + align64(kg * bhw);
    const int64_t ws_floats = scratch_floats - align64(kg * bhw);
    for (int g = 0; g < c.G; ++g) {
      add("conv2d_im2col", [=](cudaStream_t s) { launch_im2col(c, g, x, col, s); });
      GemmDesc d = base_desc(ws, ws_floats);
      d.M = opg; d.N = hwo; d.K = kg; d.batch = c.B;
      d.A = w + (int64_t)g * opg * kg; d.lda_m = kg; d.lda_k = 1; d.a_batch = 0;
      d.B = col; d.ldb_k = bhw; d.ldb_n = 1; d.b_batch = hwo;
      d.C = out + (int64_t)g * opg * hwo; d.ldc = hwo; d.c_batch = (int64_t)c.Cout * hwo;
      add(gemm_label("conv2d_gemm", d), [=](cudaStream_t s) { gemm(d, s); });
    }
  } else if (which == 1) {  // in0 = w, in1 = dy, out = dx
    const float *w = in0, *dy = in1;
    float* ws = scratch + align64(kg * bhw);
    const int64_t ws_floats = scratch_floats - align64(kg * bhw);
    for (int g = 0; g < c.G; ++g) {
      GemmDesc d = base_desc(ws, ws_floats);
      d.M = kg; d.N = hwo; d.K = opg; d.batch = c.B;
      d.A = w + (int64_t)g * opg * kg; d.lda_m = 1; d.lda_k = kg; d.a_batch = 0;
      d.B = dy + (int64_t)g * opg * hwo; d.ldb_k = hwo; d.ldb_n = 1; d.b_batch = (int64_t)c.Cout * hwo;
      d.C = col; d.ldc = bhw; d.c_batch = hwo;
      add(gemm_label("conv2d_input_grad_gemm", d), [=](cudaStream_t s) { gemm(d, s); });
      add("conv2d_input_grad_col2im", [=](cudaStream_t s) {
        if (c.kH == 3 && c.kW == 3)
          col2im_kernel<3, 3><<<row_grid((int64_t)c.B * cpg), 256, 0, s>>>(c, g, col, out);
        else
          col2im_kernel<0, 0><<<row_grid((int64_t)c.B * cpg), 256, 0, s>>>(c, g, col, out);
      });
    }
  } else {  // in0 = x, in1 = dy, out = dw
    const float *x = in0, *dy = in1;
    float* dyt = scratch + align64(kg * bhw);
    float* ws = dyt + align64((int64_t)c.Cout * bhw);
    const int64_t ws_floats = scratch_floats - align64(kg * bhw) - align64((int64_t)c.Cout * bhw);
    add("conv2d_weight_grad_swap", [=](cudaStream_t s) {
      swap_bc_kernel<<<row_grid((int64_t)c.Cout * c.B), 256, 0, s>>>(dy, dyt, c.B, c.Cout, (int)hwo);
    });
    for (int g = 0; g < c.G; ++g) {
      add("conv2d_weight_grad_im2col", [=](cudaStream_t s) {
        launch_im2col(c, g, x, col, s);
      });
      GemmDesc d = base_desc(ws, ws_floats);
      d.M = opg; d.N = kg; d.K = bhw;
      d.A = dyt + (int64_t)g * opg * bhw; d.lda_m = bhw; d.lda_k = 1;
      d.B = col; d.ldb_k = 1; d.ldb_n = bhw;
      d.C = out + (int64_t)g * opg * kg; d.ldc = kg;
      add(gemm_label("conv2d_weight_grad_gemm", d), [=](cudaStream_t s) { gemm(d, s); });
    }
  }
}

}  // namespace tg
