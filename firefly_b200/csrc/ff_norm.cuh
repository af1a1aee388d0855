// ff_norm.cuh — LayerNorm over the rows of a bf16 matrix for the BitLinear decoder, with the
// first pass of the dual int8 quantiser of its output folded in, and the column sums that give
// the LayerNorm's weight and bias gradients.
//
// Forward (one warp per row, the row held in registers as bf16x2 words):
//   mean = Σx / C,  var = Σ(x − mean)² / C,  rstd = 1 / sqrt(var + eps)       (fp32)
//   y = bf16((x − mean)·rstd·gamma + beta)
// with, on request, the row maxima of |y| and the column maxima of |y| (float bits, the
// quantiser's workspace layout: rows, then columns), after which the quantiser's second pass
// writes the row codes and the transposed column codes of y exactly as ff_quant_dual_i8 would.
// Backward (ff_layernorm_bwd, from dy, x and the saved mean and rstd): the input gradient
//   dx = bf16(rstd·(g − mean(g) − xhat·mean(g·xhat))),  g = dy·gamma,  xhat = (x − mean)·rstd
// one warp per row, and dgamma = Σ_rows dy·xhat, dbeta = Σ_rows dy by a two-stage reduction
// in a fixed order (deterministic).
#pragma once
#include "ff_common.cuh"

namespace ff {
namespace norm {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kChunk = 256;      // columns per chunk: 8 per lane
constexpr int kWgradRows = 64;   // rows per block of the weight-gradient reduction

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// MAXCH: the most 256-column chunks a row may have (cols <= 256 * MAXCH)
template <int MAXCH>
__global__ void __launch_bounds__(kThreads) ln_fwd_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                                         int64_t rows, int cols, const float* __restrict__ gamma,
                                                         const float* __restrict__ beta, float eps,
                                                         __nv_bfloat16* __restrict__ y, int64_t ldy,
                                                         float* __restrict__ mean, float* __restrict__ rstd,
                                                         uint32_t* __restrict__ row_amax,
                                                         uint32_t* __restrict__ col_amax) {
  extern __shared__ uint32_t s_colmax[];  // [cols] float bits, when the maxima are wanted
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const bool amax = row_amax != nullptr;
  if (amax)
    for (int c = threadIdx.x; c < cols; c += kThreads) s_colmax[c] = 0u;
  __syncthreads();
  uint32_t cmax[MAXCH][4];  // this lane's column maxima of |y| (bf16x2 words)
#pragma unroll
  for (int c = 0; c < MAXCH; ++c) cmax[c][0] = cmax[c][1] = cmax[c][2] = cmax[c][3] = 0u;
  const float inv_c = 1.f / (float)cols;
  for (int64_t r = (int64_t)blockIdx.x * kWarps + warp; r < rows; r += (int64_t)gridDim.x * kWarps) {
    uint32_t w[MAXCH][4];
    float s = 0.f;
#pragma unroll
    for (int c = 0; c < MAXCH; ++c) {
      const int col = c * kChunk + lane * 8;
      if (col < cols) {
        const uint4 v = *reinterpret_cast<const uint4*>(x + r * ldx + col);
        w[c][0] = v.x; w[c][1] = v.y; w[c][2] = v.z; w[c][3] = v.w;
#pragma unroll
        for (int k = 0; k < 4; ++k) s += __uint_as_float(w[c][k] << 16) + __uint_as_float(w[c][k] & 0xFFFF0000u);
      } else {
        w[c][0] = w[c][1] = w[c][2] = w[c][3] = 0u;
      }
    }
    const float mu = warp_sum(s) * inv_c;
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < MAXCH; ++c) {
      if (c * kChunk + lane * 8 < cols) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float a = __uint_as_float(w[c][k] << 16) - mu, b = __uint_as_float(w[c][k] & 0xFFFF0000u) - mu;
          ss = fmaf(a, a, ss);
          ss = fmaf(b, b, ss);
        }
      }
    }
    const float rs = 1.f / sqrtf(warp_sum(ss) * inv_c + eps);
    uint32_t rmax = 0u;
#pragma unroll
    for (int c = 0; c < MAXCH; ++c) {
      const int col = c * kChunk + lane * 8;
      if (col < cols) {
        const float4 g0 = *reinterpret_cast<const float4*>(gamma + col), g1 = *reinterpret_cast<const float4*>(gamma + col + 4);
        const float4 b0 = *reinterpret_cast<const float4*>(beta + col), b1 = *reinterpret_cast<const float4*>(beta + col + 4);
        const float gg[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
        const float bb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
        uint32_t o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float a = (__uint_as_float(w[c][k] << 16) - mu) * rs;
          const float b = (__uint_as_float(w[c][k] & 0xFFFF0000u) - mu) * rs;
          o[k] = pack_bf16x2(mk2(fmaf(a, gg[2 * k], bb[2 * k]), fmaf(b, gg[2 * k + 1], bb[2 * k + 1])));
          if (amax) {
            const uint32_t m = abs_bf16x2(o[k]);
            rmax = max_bf16x2(rmax, m);
            cmax[c][k] = max_bf16x2(cmax[c][k], m);
          }
        }
        *reinterpret_cast<uint4*>(y + r * ldy + col) = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
    if (lane == 0) {
      mean[r] = mu;
      rstd[r] = rs;
    }
    if (amax) {  // non-negative floats order like their bit patterns
      uint32_t m = max(rmax << 16, rmax & 0xFFFF0000u);
      m = __reduce_max_sync(0xffffffffu, m);
      if (lane == 0) row_amax[r] = m;
    }
  }
  if (!amax) return;
#pragma unroll
  for (int c = 0; c < MAXCH; ++c) {
    const int col = c * kChunk + lane * 8;
    if (col < cols) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        atomicMax(s_colmax + col + 2 * k, cmax[c][k] << 16);
        atomicMax(s_colmax + col + 2 * k + 1, cmax[c][k] & 0xFFFF0000u);
      }
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < cols; c += kThreads)
    if (s_colmax[c]) atomicMax(col_amax + c, s_colmax[c]);
}

// input gradient, one warp per row:  g = dy·gamma,  dx = rstd·(g − mean(g) − xhat·mean(g·xhat))
template <int MAXCH>
__global__ void __launch_bounds__(kThreads) ln_bwd_dx_kernel(const __nv_bfloat16* __restrict__ dy, int64_t lddy,
                                                            const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                                            int64_t rows, int cols, const float* __restrict__ mean,
                                                            const float* __restrict__ rstd,
                                                            const float* __restrict__ gamma,
                                                            __nv_bfloat16* __restrict__ dx, int64_t lddx) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float inv_c = 1.f / (float)cols;
  for (int64_t r = (int64_t)blockIdx.x * kWarps + warp; r < rows; r += (int64_t)gridDim.x * kWarps) {
    const float mu = __ldg(mean + r), rs = __ldg(rstd + r);
    uint32_t dw[MAXCH][4], xw[MAXCH][4];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int c = 0; c < MAXCH; ++c) {
      const int col = c * kChunk + lane * 8;
      if (col < cols) {
        const uint4 d = *reinterpret_cast<const uint4*>(dy + r * lddy + col);
        const uint4 v = *reinterpret_cast<const uint4*>(x + r * ldx + col);
        dw[c][0] = d.x; dw[c][1] = d.y; dw[c][2] = d.z; dw[c][3] = d.w;
        xw[c][0] = v.x; xw[c][1] = v.y; xw[c][2] = v.z; xw[c][3] = v.w;
        const float4 g0 = *reinterpret_cast<const float4*>(gamma + col), g1 = *reinterpret_cast<const float4*>(gamma + col + 4);
        const float gg[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float ga = __uint_as_float(dw[c][k] << 16) * gg[2 * k];
          const float gb = __uint_as_float(dw[c][k] & 0xFFFF0000u) * gg[2 * k + 1];
          const float xa = (__uint_as_float(xw[c][k] << 16) - mu) * rs;
          const float xb = (__uint_as_float(xw[c][k] & 0xFFFF0000u) - mu) * rs;
          s1 += ga + gb;
          s2 = fmaf(ga, xa, fmaf(gb, xb, s2));
        }
      }
    }
    const float c1 = warp_sum(s1) * inv_c, c2 = warp_sum(s2) * inv_c;
#pragma unroll
    for (int c = 0; c < MAXCH; ++c) {
      const int col = c * kChunk + lane * 8;
      if (col < cols) {
        const float4 g0 = *reinterpret_cast<const float4*>(gamma + col), g1 = *reinterpret_cast<const float4*>(gamma + col + 4);
        const float gg[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
        uint32_t o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float ga = __uint_as_float(dw[c][k] << 16) * gg[2 * k];
          const float gb = __uint_as_float(dw[c][k] & 0xFFFF0000u) * gg[2 * k + 1];
          const float xa = (__uint_as_float(xw[c][k] << 16) - mu) * rs;
          const float xb = (__uint_as_float(xw[c][k] & 0xFFFF0000u) - mu) * rs;
          o[k] = pack_bf16x2(mk2(rs * (ga - c1 - xa * c2), rs * (gb - c1 - xb * c2)));
        }
        *reinterpret_cast<uint4*>(dx + r * lddx + col) = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  }
}

// stage 1: per block of kWgradRows rows, the column sums of dy·xhat and dy (8 columns per thread)
__global__ void __launch_bounds__(kThreads) ln_wgrad_stage1(const __nv_bfloat16* __restrict__ dy, int64_t lddy,
                                                           const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                                           int64_t rows, int cols, const float* __restrict__ mean,
                                                           const float* __restrict__ rstd, float* __restrict__ ws) {
  const int64_t rb = blockIdx.y;
  const int col = (blockIdx.x * kThreads + threadIdx.x) * 8;
  if (col >= cols) return;
  float ag[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, ab[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  const int64_t r0 = rb * kWgradRows, r1 = min64(rows, r0 + kWgradRows);
  for (int64_t r = r0; r < r1; ++r) {
    const float mu = __ldg(mean + r), rs = __ldg(rstd + r);
    const uint4 d = *reinterpret_cast<const uint4*>(dy + r * lddy + col);
    const uint4 v = *reinterpret_cast<const uint4*>(x + r * ldx + col);
    const uint32_t dw[4] = {d.x, d.y, d.z, d.w}, xw[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float d0 = __uint_as_float(dw[k] << 16), d1 = __uint_as_float(dw[k] & 0xFFFF0000u);
      const float x0 = (__uint_as_float(xw[k] << 16) - mu) * rs, x1 = (__uint_as_float(xw[k] & 0xFFFF0000u) - mu) * rs;
      ag[2 * k] = fmaf(d0, x0, ag[2 * k]);
      ag[2 * k + 1] = fmaf(d1, x1, ag[2 * k + 1]);
      ab[2 * k] += d0;
      ab[2 * k + 1] += d1;
    }
  }
  float* wg = ws + (size_t)rb * 2 * cols;
  *reinterpret_cast<float4*>(wg + col) = make_float4(ag[0], ag[1], ag[2], ag[3]);
  *reinterpret_cast<float4*>(wg + col + 4) = make_float4(ag[4], ag[5], ag[6], ag[7]);
  *reinterpret_cast<float4*>(wg + cols + col) = make_float4(ab[0], ab[1], ab[2], ab[3]);
  *reinterpret_cast<float4*>(wg + cols + col + 4) = make_float4(ab[4], ab[5], ab[6], ab[7]);
}

// stage 2: per column, the row blocks' partial sums in a fixed order: warp w of the CTA adds the
// w-th eighth of the blocks in block order, then the eight range sums are added in warp order.
// A CTA takes 32 columns of dgamma (blockIdx.y = 0) or dbeta (1); a warp reads 128 B per block.
constexpr int kS2Cols = 32;
__global__ void __launch_bounds__(kThreads) ln_wgrad_stage2(const float* __restrict__ ws, int64_t nblocks, int cols,
                                                           float* __restrict__ dgamma, float* __restrict__ dbeta) {
  constexpr int kSlices = kThreads / kS2Cols;
  __shared__ float part[kSlices][kS2Cols];
  const int lane = threadIdx.x % kS2Cols, slice = threadIdx.x / kS2Cols;
  const int c = blockIdx.x * kS2Cols + lane;
  float* out = blockIdx.y == 0 ? dgamma : dbeta;
  if (out == nullptr) return;  // uniform over the CTA
  const int64_t per = (nblocks + kSlices - 1) / kSlices;
  const int64_t k0 = min64(nblocks, slice * per), k1 = min64(nblocks, k0 + per);
  float acc = 0.f;
  if (c < cols) {
    const float* src = ws + (blockIdx.y == 0 ? 0 : cols) + c;
    for (int64_t k = k0; k < k1; ++k) acc += src[(size_t)k * 2 * cols];
  }
  part[slice][lane] = acc;
  __syncthreads();
  if (slice == 0 && c < cols) {
    float t = part[0][lane];
#pragma unroll
    for (int s = 1; s < kSlices; ++s) t += part[s][lane];
    out[c] = t;
  }
}

template <int MAXCH>
inline void launch_ln_fwd(int grid, size_t smem, cudaStream_t st, const __nv_bfloat16* x, int64_t ldx, int64_t rows,
                          int cols, const float* gamma, const float* beta, float eps, __nv_bfloat16* y, int64_t ldy,
                          float* mean, float* rstd, uint32_t* row_amax, uint32_t* col_amax) {
  ln_fwd_kernel<MAXCH><<<grid, kThreads, smem, st>>>(x, ldx, rows, cols, gamma, beta, eps, y, ldy, mean, rstd,
                                                     row_amax, col_amax);
}

}  // namespace norm
}  // namespace ff

extern "C" int ff_layernorm_i8(const uint16_t* x, int64_t ldx, int64_t rows, int64_t cols, const float* gamma,
                               const float* beta, float eps, uint16_t* y, int64_t ldy, float* mean, float* rstd,
                               float q_eps, int8_t* q_rows, int64_t ldq, float* s_rows, int8_t* q_cols_t,
                               int64_t ldqt, float* s_cols, float* absmax_ws, void* stream) {
  using namespace ff;
  using namespace ff::norm;
  const char* name = "ff_layernorm_i8";
  FF_REQUIRE(rows >= 0 && cols >= 8 && ldx >= cols && ldy >= cols, FF_ERR_INVALID_ARG,
             "%s: rows=%lld cols=%lld ldx=%lld ldy=%lld", name, (long long)rows, (long long)cols, (long long)ldx,
             (long long)ldy);
  FF_REQUIRE(cols % 8 == 0 && cols <= 16 * kChunk && ldx % 8 == 0 && ldy % 8 == 0, FF_ERR_UNSUPPORTED,
             "%s: cols must be a multiple of 8 up to %d, leading dims multiples of 8", name, 16 * kChunk);
  if (rows == 0) return FF_OK;
  FF_REQUIRE(x && gamma && beta && y && mean && rstd, FF_ERR_INVALID_ARG, "%s: null pointer", name);
  FF_REQUIRE(aligned(x, 16) && aligned(y, 16) && aligned(gamma, 16) && aligned(beta, 16), FF_ERR_UNSUPPORTED,
             "%s: x, y, gamma and beta need 16-byte alignment", name);
  const bool quant = q_rows || q_cols_t;
  cudaStream_t st = as_stream(stream);
  if (quant) {
    const int rc = check_dual_outputs(name, rows, cols, q_rows, ldq, s_rows, q_cols_t, ldqt, s_cols, absmax_ws);
    if (rc != FF_OK) return rc;
    FF_CUDA_TRY(cudaMemsetAsync(absmax_ws, 0, sizeof(float) * (size_t)(rows + cols), st), name);
  }
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = (int)min64((rows + kWarps - 1) / kWarps, (int64_t)sms * 8);
  const size_t smem = quant ? sizeof(uint32_t) * (size_t)cols : 0;
  uint32_t* ra = quant ? reinterpret_cast<uint32_t*>(absmax_ws) : nullptr;
  uint32_t* ca = quant ? ra + rows : nullptr;
  const auto* xb = reinterpret_cast<const __nv_bfloat16*>(x);
  auto* yb = reinterpret_cast<__nv_bfloat16*>(y);
  if (cols <= 8 * kChunk)
    launch_ln_fwd<8>(grid, smem, st, xb, ldx, rows, (int)cols, gamma, beta, eps, yb, ldy, mean, rstd, ra, ca);
  else
    launch_ln_fwd<16>(grid, smem, st, xb, ldx, rows, (int)cols, gamma, beta, eps, yb, ldy, mean, rstd, ra, ca);
  if (!quant) return check_launch(name);
  const int rc = check_launch(name);
  if (rc != FF_OK) return rc;
  return launch_pass_b<FF_DTYPE_BF16>(name, yb, rows, cols, ldy, nullptr, q_eps, q_rows, ldq, s_rows, q_cols_t, ldqt,
                                      s_cols, absmax_ws, st);
}

extern "C" int64_t ff_layernorm_bwd_ws_elems(int64_t rows, int64_t cols) {
  using namespace ff::norm;
  return 2 * cols * ((rows + kWgradRows - 1) / kWgradRows);
}

extern "C" int ff_layernorm_bwd(const uint16_t* dy, int64_t lddy, const uint16_t* x, int64_t ldx, int64_t rows,
                                int64_t cols, const float* mean, const float* rstd, const float* gamma, uint16_t* dx,
                                int64_t lddx, float* dgamma, float* dbeta, float* ws, void* stream) {
  using namespace ff;
  using namespace ff::norm;
  const char* name = "ff_layernorm_bwd";
  FF_REQUIRE(rows >= 0 && cols >= 8 && lddy >= cols && ldx >= cols && (!dx || lddx >= cols), FF_ERR_INVALID_ARG,
             "%s: bad sizes", name);
  FF_REQUIRE(cols % 8 == 0 && lddy % 8 == 0 && ldx % 8 == 0 && (!dx || lddx % 8 == 0), FF_ERR_UNSUPPORTED,
             "%s: cols and leading dims must be multiples of 8", name);
  FF_REQUIRE(!dx || cols <= 16 * kChunk, FF_ERR_UNSUPPORTED, "%s: cols must be at most %d for dx", name,
             16 * kChunk);
  FF_REQUIRE(dx || dgamma || dbeta, FF_ERR_INVALID_ARG, "%s: nothing to do", name);
  cudaStream_t st = as_stream(stream);
  if (rows == 0) {
    if (dgamma) FF_CUDA_TRY(cudaMemsetAsync(dgamma, 0, sizeof(float) * (size_t)cols, st), name);
    if (dbeta) FF_CUDA_TRY(cudaMemsetAsync(dbeta, 0, sizeof(float) * (size_t)cols, st), name);
    return FF_OK;
  }
  FF_REQUIRE(dy && x && mean && rstd && (!dx || gamma) && (!(dgamma || dbeta) || ws), FF_ERR_INVALID_ARG,
             "%s: null pointer", name);
  FF_REQUIRE(aligned(dy, 16) && aligned(x, 16) && (!dx || (aligned(dx, 16) && aligned(gamma, 16))) &&
                 (!ws || aligned(ws, 16)),
             FF_ERR_UNSUPPORTED, "%s: dy, x, dx, gamma and ws need 16-byte alignment", name);
  const auto* dyb = reinterpret_cast<const __nv_bfloat16*>(dy);
  const auto* xb = reinterpret_cast<const __nv_bfloat16*>(x);
  if (dx) {
    int sms = 148, dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int grid = (int)min64((rows + kWarps - 1) / kWarps, (int64_t)sms * 8);
    auto* dxb = reinterpret_cast<__nv_bfloat16*>(dx);
    if (cols <= 8 * kChunk)
      ln_bwd_dx_kernel<8><<<grid, kThreads, 0, st>>>(dyb, lddy, xb, ldx, rows, (int)cols, mean, rstd, gamma, dxb, lddx);
    else
      ln_bwd_dx_kernel<16><<<grid, kThreads, 0, st>>>(dyb, lddy, xb, ldx, rows, (int)cols, mean, rstd, gamma, dxb,
                                                      lddx);
  }
  if (dgamma || dbeta) {
    const int64_t nb = (rows + kWgradRows - 1) / kWgradRows;
    FF_REQUIRE(nb < 65536, FF_ERR_UNSUPPORTED, "%s: too many rows", name);
    const dim3 g1((unsigned)((cols / 8 + kThreads - 1) / kThreads), (unsigned)nb);
    ln_wgrad_stage1<<<g1, kThreads, 0, st>>>(dyb, lddy, xb, ldx, rows, (int)cols, mean, rstd, ws);
    ln_wgrad_stage2<<<dim3((unsigned)((cols + kS2Cols - 1) / kS2Cols), 2), kThreads, 0, st>>>(ws, nb, (int)cols,
                                                                                              dgamma, dbeta);
  }
  return check_launch(name);
}
