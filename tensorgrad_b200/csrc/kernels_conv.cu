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
#include "kernels.cuh"

namespace tg {

static unsigned conv_grid(int64_t work) {
  int64_t b = (work + 255) / 256;
  int64_t cap = (int64_t)device_sm_count() * 16;
  if (b > cap) b = cap;
  if (b < 1) b = 1;
  return (unsigned)b;
}

__global__ void __launch_bounds__(256) im2col_kernel(const __grid_constant__ ConvDesc c, int g,
                                                     const float* __restrict__ x, float* __restrict__ col) {
  const int cpg = c.Cin / c.G, kk = c.kH * c.kW, hwo = c.Hout * c.Wout;
  const int64_t bhw = (int64_t)c.B * hwo;
  const int64_t total = (int64_t)cpg * kk * bhw;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int k = (int)(i / bhw);
    const int64_t r = i - (int64_t)k * bhw;
    const int b = (int)(r / hwo);
    const int p = (int)(r - (int64_t)b * hwo);
    const int ho = p / c.Wout, wo = p - ho * c.Wout;
    const int cl = k / kk, kr = k - cl * kk;
    const int kh = kr / c.kW, kw = kr - kh * c.kW;
    const int hi = ho * c.sH + kh - c.pH, wi = wo * c.sW + kw - c.pW;
    float v = 0.f;
    if (hi >= 0 && hi < c.H && wi >= 0 && wi < c.W)
      v = x[(((int64_t)b * c.Cin + g * cpg + cl) * c.H + hi) * c.W + wi];
    col[i] = v;
  }
}

// dx[b, g*cpg + cl, h, w] = sum of dcol over the (kh, kw) taps whose output
// position lands on (h, w); taps in ascending (kh, kw) order.
__global__ void __launch_bounds__(256) col2im_kernel(const __grid_constant__ ConvDesc c, int g,
                                                     const float* __restrict__ dcol, float* __restrict__ dx) {
  const int cpg = c.Cin / c.G, kk = c.kH * c.kW, hwo = c.Hout * c.Wout;
  const int64_t bhw = (int64_t)c.B * hwo;
  const int64_t total = (int64_t)c.B * cpg * c.H * c.W;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int wi = (int)(i % c.W);
    const int hi = (int)((i / c.W) % c.H);
    const int cl = (int)((i / ((int64_t)c.W * c.H)) % cpg);
    const int b = (int)(i / ((int64_t)c.W * c.H * cpg));
    float s = 0.f;
    for (int kh = 0; kh < c.kH; ++kh) {
      const int nh = hi + c.pH - kh;
      if (nh < 0 || nh % c.sH) continue;
      const int ho = nh / c.sH;
      if (ho >= c.Hout) continue;
      for (int kw = 0; kw < c.kW; ++kw) {
        const int nw = wi + c.pW - kw;
        if (nw < 0 || nw % c.sW) continue;
        const int wo = nw / c.sW;
        if (wo >= c.Wout) continue;
        s += dcol[(int64_t)(cl * kk + kh * c.kW + kw) * bhw + (int64_t)b * hwo + ho * c.Wout + wo];
      }
    }
    dx[(((int64_t)b * c.Cin + g * cpg + cl) * c.H + hi) * c.W + wi] = s;
  }
}

// dyT[ch, b*hw + p] = dy[b, ch, p]: contiguous runs of hw floats move whole.
__global__ void __launch_bounds__(256) swap_bc_kernel(const float* __restrict__ dy, float* __restrict__ dyt,
                                                      int B, int C, int hw) {
  const int64_t total = (int64_t)B * C * hw;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int p = (int)(i % hw);
    const int64_t bc = i / hw;
    const int ch = (int)(bc % C), b = (int)(bc / C);
    dyt[((int64_t)ch * B + b) * hw + p] = dy[i];
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

void launch_conv2d_gemm(const ConvDesc& c, const float* x, const float* w, float* y, float* scratch,
                        int64_t scratch_floats, cudaStream_t s) {
  const int cpg = c.Cin / c.G, opg = c.Cout / c.G;
  const int64_t kg = (int64_t)cpg * c.kH * c.kW, hwo = (int64_t)c.Hout * c.Wout, bhw = c.B * hwo;
  float* col = scratch;
  float* ws = scratch + align64(kg * bhw);
  const int64_t ws_floats = scratch_floats - align64(kg * bhw);
  for (int g = 0; g < c.G; ++g) {
    im2col_kernel<<<conv_grid(kg * bhw), 256, 0, s>>>(c, g, x, col);
    GemmDesc d = base_desc(ws, ws_floats);
    d.M = opg; d.N = hwo; d.K = kg; d.batch = c.B;
    d.A = w + (int64_t)g * opg * kg; d.lda_m = kg; d.lda_k = 1; d.a_batch = 0;
    d.B = col; d.ldb_k = bhw; d.ldb_n = 1; d.b_batch = hwo;
    d.C = y + (int64_t)g * opg * hwo; d.ldc = hwo; d.c_batch = (int64_t)c.Cout * hwo;
    gemm(d, s);
  }
}

void launch_conv2d_input_grad_gemm(const ConvDesc& c, const float* w, const float* dy, float* dx, float* scratch,
                                   int64_t scratch_floats, cudaStream_t s) {
  const int cpg = c.Cin / c.G, opg = c.Cout / c.G;
  const int64_t kg = (int64_t)cpg * c.kH * c.kW, hwo = (int64_t)c.Hout * c.Wout, bhw = c.B * hwo;
  float* dcol = scratch;
  float* ws = scratch + align64(kg * bhw);
  const int64_t ws_floats = scratch_floats - align64(kg * bhw);
  for (int g = 0; g < c.G; ++g) {
    GemmDesc d = base_desc(ws, ws_floats);
    d.M = kg; d.N = hwo; d.K = opg; d.batch = c.B;
    d.A = w + (int64_t)g * opg * kg; d.lda_m = 1; d.lda_k = kg; d.a_batch = 0;
    d.B = dy + (int64_t)g * opg * hwo; d.ldb_k = hwo; d.ldb_n = 1; d.b_batch = (int64_t)c.Cout * hwo;
    d.C = dcol; d.ldc = bhw; d.c_batch = hwo;
    gemm(d, s);
    col2im_kernel<<<conv_grid((int64_t)c.B * cpg * c.H * c.W), 256, 0, s>>>(c, g, dcol, dx);
  }
}

void launch_conv2d_weight_grad_gemm(const ConvDesc& c, const float* x, const float* dy, float* dw, float* scratch,
                                    int64_t scratch_floats, cudaStream_t s) {
  const int cpg = c.Cin / c.G, opg = c.Cout / c.G;
  const int64_t kg = (int64_t)cpg * c.kH * c.kW, hwo = (int64_t)c.Hout * c.Wout, bhw = c.B * hwo;
  float* col = scratch;
  float* dyt = scratch + align64(kg * bhw);
  float* ws = dyt + align64((int64_t)c.Cout * bhw);
  const int64_t ws_floats = scratch_floats - align64(kg * bhw) - align64((int64_t)c.Cout * bhw);
  swap_bc_kernel<<<conv_grid((int64_t)c.Cout * bhw), 256, 0, s>>>(dy, dyt, c.B, c.Cout, (int)hwo);
  for (int g = 0; g < c.G; ++g) {
    im2col_kernel<<<conv_grid(kg * bhw), 256, 0, s>>>(c, g, x, col);
    GemmDesc d = base_desc(ws, ws_floats);
    d.M = opg; d.N = kg; d.K = bhw;
    d.A = dyt + (int64_t)g * opg * bhw; d.lda_m = bhw; d.lda_k = 1;
    d.B = col; d.ldb_k = 1; d.ldb_n = bhw;
    d.C = dw + (int64_t)g * opg * kg; d.ldc = kg;
    gemm(d, s);
  }
}

}  // namespace tg
