// ff_gelu.cuh — the tanh form of GELU and its derivative, as the fused GEMM epilogues of a
// BitLinear GELU MLP evaluate them.
//
//   gelu(x)  = 0.5·x·(1 + tanh(b·(x + k·x³))),            b = sqrt(2/pi), k = 0.044715
//   gelu'(x) = 0.5·(1 + t) + 0.5·x·(1 − t²)·b·(1 + 3k·x²),  t = tanh(b·(x + k·x³))
//
// computed in fp32 from a bf16 input with tanhf, each operation rounded once, in the order of
// the usual elementwise formulation (x³ = (x·x)·x; the backward forms x² first).  Where a
// compiler may contract a multiply and an add into one FMA, the variant bits choose:
//   1: forward  x + k·x³ as fma(k, x³, x)          16: the same in the backward
//   2: 1 − t·t as fma(−t, t, 1)                     4: 1 + 3k·x² as fma(3k, x², 1)
//   8: the final sum 0.5·(1 + t) + P·Q as fma(P, Q, 0.5·(1 + t))
//  32: the product order of the derivative's second term: P·Q = ((0.5·x)·(1 − t²))·(b·(1 + 3k·x²))
//      without it, (((0.5·x)·(1 − t²))·b)·(1 + 3k·x²)
// The host picks, once per device, the variant whose results equal torch's GELU kernels for
// all 65536 bf16 inputs (ff_gelu_eval returns both functions for a list of inputs).
#pragma once
#include <cmath>

#include "ff_common.cuh"

namespace ff {
namespace gelu {

constexpr float kBeta = (float)(M_SQRT2 * M_2_SQRTPI * 0.5);
constexpr float kKappa = 0.044715f;
constexpr float k3Kappa = 3.0f * kKappa;  // the fp32 product

__device__ __forceinline__ float inner(float x, float x3, bool fused) {
  const float s = fused ? __fmaf_rn(kKappa, x3, x) : __fadd_rn(x, __fmul_rn(kKappa, x3));
  return __fmul_rn(kBeta, s);
}

__device__ __forceinline__ float fwd(float x, int v) {
  const float x3 = __fmul_rn(__fmul_rn(x, x), x);
  const float t = tanhf(inner(x, x3, v & 1));
  return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.f, t));
}

__device__ __forceinline__ float grad(float x, int v) {
  const float x2 = __fmul_rn(x, x);
  const float x3 = __fmul_rn(x2, x);
  const float t = tanhf(inner(x, x3, v & 16));
  const float ld = __fmul_rn(0.5f, __fadd_rn(1.f, t));
  const float q = (v & 2) ? __fmaf_rn(-t, t, 1.f) : __fsub_rn(1.f, __fmul_rn(t, t));
  const float p = (v & 4) ? __fmaf_rn(k3Kappa, x2, 1.f) : __fadd_rn(1.f, __fmul_rn(k3Kappa, x2));
  const float lq = __fmul_rn(__fmul_rn(0.5f, x), q);
  const float P = (v & 32) ? lq : __fmul_rn(lq, kBeta);
  const float Q = (v & 32) ? __fmul_rn(kBeta, p) : p;
  return (v & 8) ? __fmaf_rn(P, Q, ld) : __fadd_rn(ld, __fmul_rn(P, Q));
}

__global__ void eval_kernel(const uint16_t* x, int64_t n, int fv, int bv, float* h, float* d) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float xf = __uint_as_float((uint32_t)x[i] << 16);
    if (h) h[i] = fwd(xf, fv);
    if (d) d[i] = grad(xf, bv);
  }
}

}  // namespace gelu
}  // namespace ff

extern "C" int ff_gelu_eval(const uint16_t* x, int64_t n, int fwd_variant, int bwd_variant, float* h, float* d,
                            void* stream) {
  using namespace ff;
  FF_REQUIRE(n >= 0 && fwd_variant >= 0 && fwd_variant < 64 && bwd_variant >= 0 && bwd_variant < 64,
             FF_ERR_INVALID_ARG, "ff_gelu_eval: n=%lld variants %d/%d", (long long)n, fwd_variant, bwd_variant);
  if (n == 0) return FF_OK;
  FF_REQUIRE(x && (h || d), FF_ERR_INVALID_ARG, "ff_gelu_eval: null pointer");
  const int grid = (int)min64((n + 255) / 256, 1024);
  gelu::eval_kernel<<<grid, 256, 0, as_stream(stream)>>>(x, n, fwd_variant, bwd_variant, h, d);
  return check_launch("ff_gelu_eval");
}
