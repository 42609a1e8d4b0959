// Elementwise program kernel: evaluates a fused straight-line program of
// elementwise IR ops over every output element. In the reference each of
// these ops is its own WGSL kernel (src/codegen.ts:107-330 arithmetic,
// compare/select and relu_grad, :241-268 dropout, :691-712 where_causal,
// :841-905 Adam).
//
// B200 design: the work is HBM-bound, so each thread handles 4 consecutive
// elements with 128-bit loads/stores when every operand allows it; the grid is
// a multiple of the SM count and walks the tensor grid-stride. The program
// lives in the kernel parameter block (constant bank) and every thread runs
// the same instruction stream, so dispatch never diverges. Registers are a
// fixed file of EW_NREG values per lane accessed through compile-time
// switches, which keeps them in hardware registers.
#include "kernels.cuh"

namespace tg {

int device_sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (!cached[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

template <int V>
struct RegFile {
  float r[EW_NREG][V];
};

template <int V>
__device__ __forceinline__ void rget(const RegFile<V>& R, int i, float (&o)[V]) {
#define RG_CASE(k) case k: _Pragma("unroll") for (int l = 0; l < V; ++l) o[l] = R.r[k][l]; break;
  switch (i) { RG_CASE(0) RG_CASE(1) RG_CASE(2) RG_CASE(3) RG_CASE(4) RG_CASE(5) RG_CASE(6) RG_CASE(7) }
#undef RG_CASE
}

template <int V>
__device__ __forceinline__ void rset(RegFile<V>& R, int i, const float (&o)[V]) {
#define RS_CASE(k) case k: _Pragma("unroll") for (int l = 0; l < V; ++l) R.r[k][l] = o[l]; break;
  switch (i) { RS_CASE(0) RS_CASE(1) RS_CASE(2) RS_CASE(3) RS_CASE(4) RS_CASE(5) RS_CASE(6) RS_CASE(7) }
#undef RS_CASE
}

// PCG output permutation on u32, the reference's stochastic hash
// (src/codegen.ts:224-227).
__device__ __forceinline__ uint32_t pcg(uint32_t h) {
  h = h * 747796405u + 2891336453u;
  h = ((h >> ((h >> 28u) + 4u)) ^ h) * 277803737u;
  return (h >> 22u) ^ h;
}

// erf by Abramowitz & Stegun 7.1.26, the method the reference specifies for
// its erf op (src/codegen.ts:189-197, test/_eval.ts:193-198).
__device__ __forceinline__ float erf_as(float x) {
  float s = x > 0.f ? 1.f : (x < 0.f ? -1.f : 0.f);
  float ax = fabsf(x);
  float t = 1.0f / (1.0f + 0.3275911f * ax);
  float p = t * (0.254829592f + t * (-0.284496736f + t * (1.421413741f + t * (-1.453152027f + t * 1.061405429f))));
  return s * (1.0f - p * expf(-ax * ax));
}

__device__ __forceinline__ int64_t in_offset(const EwInput& in, const EwProgram& P, int64_t i) {
  switch (in.mode) {
    case IN_FULL: return i;
    case IN_SCALAR: return 0;
    case IN_PERIOD: return i % in.period;
    case IN_ROWDIV: return i / in.period;
    default: {
      int64_t off = 0, rem = i;
      for (int d = P.rank - 1; d >= 0; --d) {
        int64_t c = rem % P.dims[d];
        rem /= P.dims[d];
        off += c * in.strides[d];
      }
      return off;
    }
  }
}

template <int V>
__device__ __forceinline__ void load_input(const EwInput& in, const EwProgram& P, int64_t i, float (&o)[V]) {
  const float* base = reinterpret_cast<const float*>(in.ptr);
  if (in.mode == IN_ONEHOT) {
    const int* ix = reinterpret_cast<const int*>(in.ptr);
#pragma unroll
    for (int l = 0; l < V; ++l) {
      int64_t e = i + l;
      o[l] = (int64_t)__ldg(ix + e / in.period) == e % in.period ? 1.f : 0.f;
    }
  } else if (in.mode == IN_SCALAR) {
    float s = __ldg(base);
#pragma unroll
    for (int l = 0; l < V; ++l) o[l] = s;
  } else if (V == 4 && in.mode == IN_ROWDIV) {
    // 4 consecutive elements share one row (period % 4 == 0 on this path)
    float s = __ldg(base + i / in.period);
#pragma unroll
    for (int l = 0; l < V; ++l) o[l] = s;
  } else if (V == 4) {
    float4 q = __ldg(reinterpret_cast<const float4*>(base + in_offset(in, P, i)));
    o[0] = q.x; o[1] = q.y; o[2] = q.z; o[3] = q.w;
  } else {
#pragma unroll
    for (int l = 0; l < V; ++l) o[l] = __ldg(base + in_offset(in, P, i + l));
  }
}

template <int V>
__device__ __forceinline__ void run_program(const EwProgram& P, int64_t i, uint32_t seed) {
  RegFile<V> R;
  for (int pc = 0; pc < P.n_instr; ++pc) {
    const EwInstr& I = P.code[pc];
    float a[V], b[V], c[V], o[V];
    if (I.op == EW_LOAD) {
      load_input<V>(P.in[I.a], P, i, o);
      rset<V>(R, I.dst, o);
      continue;
    }
    if (I.op == EW_CONST) {
      float cv = I.c ? __int_as_float((int)I.aux) : I.imm;
      for (int l = 0; l < V; ++l) o[l] = cv;
      rset<V>(R, I.dst, o);
      continue;
    }
    rget<V>(R, I.a, a);
    switch (I.op) {
      case EW_ADD: rget<V>(R, I.b, b); for (int l = 0; l < V; ++l) o[l] = a[l] + b[l]; break;
      case EW_SUB: rget<V>(R, I.b, b); for (int l = 0; l < V; ++l) o[l] = a[l] - b[l]; break;
      case EW_MUL: rget<V>(R, I.b, b); for (int l = 0; l < V; ++l) o[l] = a[l] * b[l]; break;
      case EW_DIV: rget<V>(R, I.b, b); for (int l = 0; l < V; ++l) o[l] = __fdiv_rn(a[l], b[l]); break;
      case EW_MIN: rget<V>(R, I.b, b); for (int l = 0; l < V; ++l) o[l] = fminf(a[l], b[l]); break;
      case EW_MAX: rget<V>(R, I.b, b); for (int l = 0; l < V; ++l) o[l] = fmaxf(a[l], b[l]); break;
      case EW_MULS: for (int l = 0; l < V; ++l) o[l] = a[l] * I.imm; break;
      case EW_ADDS: for (int l = 0; l < V; ++l) o[l] = a[l] + I.imm; break;
      case EW_SQRT: for (int l = 0; l < V; ++l) o[l] = __fsqrt_rn(a[l]); break;
      case EW_RSQRT: for (int l = 0; l < V; ++l) o[l] = __fdiv_rn(1.0f, __fsqrt_rn(a[l])); break;
      case EW_LOG: for (int l = 0; l < V; ++l) o[l] = logf(a[l]); break;
      case EW_EXP: for (int l = 0; l < V; ++l) o[l] = expf(a[l]); break;
      case EW_RELU: for (int l = 0; l < V; ++l) o[l] = fmaxf(a[l], 0.f); break;
      case EW_NEG: for (int l = 0; l < V; ++l) o[l] = -a[l]; break;
      case EW_ABS: for (int l = 0; l < V; ++l) o[l] = fabsf(a[l]); break;
      case EW_TANH: for (int l = 0; l < V; ++l) o[l] = tanhf(a[l]); break;
      case EW_SIGMOID: for (int l = 0; l < V; ++l) o[l] = 0.5f + 0.5f * tanhf(0.5f * a[l]); break;
      case EW_ERF: for (int l = 0; l < V; ++l) o[l] = erf_as(a[l]); break;
      case EW_SIN: for (int l = 0; l < V; ++l) o[l] = sinf(a[l]); break;
      case EW_COS: for (int l = 0; l < V; ++l) o[l] = cosf(a[l]); break;
      case EW_LESS:
        rget<V>(R, I.b, b);
        for (int l = 0; l < V; ++l) {
          bool t = I.aux ? (__float_as_int(a[l]) < __float_as_int(b[l])) : (a[l] < b[l]);
          o[l] = __int_as_float(t ? 1 : 0);
        }
        break;
      case EW_GREATER:
        rget<V>(R, I.b, b);
        for (int l = 0; l < V; ++l) {
          bool t = I.aux ? (__float_as_int(a[l]) > __float_as_int(b[l])) : (a[l] > b[l]);
          o[l] = __int_as_float(t ? 1 : 0);
        }
        break;
      case EW_WHERE:
        rget<V>(R, I.b, b); rget<V>(R, I.c, c);
        for (int l = 0; l < V; ++l) o[l] = __float_as_int(a[l]) != 0 ? b[l] : c[l];
        break;
      case EW_RELU_GRAD:
        rget<V>(R, I.b, b);
        for (int l = 0; l < V; ++l) o[l] = a[l] > 0.f ? b[l] : 0.f;
        break;
      case EW_DROPOUT:
        for (int l = 0; l < V; ++l) {
          uint32_t idx = (uint32_t)(P.drop_offset + i + l);
          uint32_t h = pcg(seed ^ I.aux ^ idx);
          float u = __uint2float_rn(h) * 2.3283064365386963e-10f;  // exact divide by 2^32
          o[l] = a[l] * (u >= I.imm ? I.imm2 : 0.f);
        }
        break;
      case EW_WHERE_CAUSAL: {
        int64_t T = I.aux;
        for (int l = 0; l < V; ++l) {
          int64_t e = i + l;
          int64_t kk = e % T, q = (e / T) % T;
          o[l] = kk > q ? I.imm : a[l];
        }
        break;
      }
      case EW_ADAM_M:
        rget<V>(R, I.b, b);
        for (int l = 0; l < V; ++l) o[l] = I.imm * a[l] + I.imm2 * b[l];
        break;
      case EW_ADAM_V:
        rget<V>(R, I.b, b);
        for (int l = 0; l < V; ++l) o[l] = I.imm * a[l] + I.imm2 * b[l] * b[l];
        break;
      case EW_ADAM_P: {
        float lr[V], sh[V], vv[V];
        rget<V>(R, I.b, b); rget<V>(R, I.c, lr); rget<V>(R, I.d, sh); rget<V>(R, I.e, vv);
        for (int l = 0; l < V; ++l) o[l] = sh[l] * a[l] - __fdiv_rn(lr[l] * b[l], __fsqrt_rn(vv[l]) + I.imm);
        break;
      }
      case EW_COPY: for (int l = 0; l < V; ++l) o[l] = a[l]; break;
      default: for (int l = 0; l < V; ++l) o[l] = 0.f; break;
    }
    rset<V>(R, I.dst, o);
  }
  for (int k = 0; k < P.n_out; ++k) {
    float o[V];
    rget<V>(R, P.out_reg[k], o);
    float* dst = reinterpret_cast<float*>(P.out[k]) + i;
    if (V == 4) {
      *reinterpret_cast<float4*>(dst) = make_float4(o[0], o[1], o[2], o[3]);
    } else {
#pragma unroll
      for (int l = 0; l < V; ++l) dst[l] = o[l];
    }
  }
}

template <int V>
__global__ void __launch_bounds__(256) ew_kernel(const __grid_constant__ EwProgram P) {
  uint32_t seed = P.seed ? (uint32_t)(*P.seed) : 0u;
  int64_t nv = P.numel / V;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < nv; t += stride) {
    run_program<V>(P, t * V, seed);
  }
}

void launch_ew(const EwProgram& p, cudaStream_t s) {
  if (p.numel <= 0) return;
  const int threads = 256;
  int V = p.vec4 ? 4 : 1;
  int64_t work = p.numel / V;
  int64_t blocks = (work + threads - 1) / threads;
  int64_t cap = (int64_t)device_sm_count() * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  if (V == 4) ew_kernel<4><<<(unsigned)blocks, threads, 0, s>>>(p);
  else ew_kernel<1><<<(unsigned)blocks, threads, 0, s>>>(p);
}

}  // namespace tg
