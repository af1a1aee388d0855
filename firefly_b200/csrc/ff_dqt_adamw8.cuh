// ff_dqt_adamw8.cuh — fused DQT-SR 8-bit AdamW update of int8 weights (one HBM pass).
//
// Replaces the per-module body of FireFlyOptim.step (fireflyoptim.py:137-209):
// ~40 torch elementwise passes plus a host sync become one kernel that reads
// g (bf16), q (int8), the m/v/r uint8 codes and their block absmax, and
// writes q, the codes and the new absmax.
//
// Work split: one warp per 256-element block, 8 consecutive elements per lane
// (16 B of g, 8 B of each code array per lane: fully coalesced).  The block
// absmax of the re-encoded r, m, v is a warp max-reduction.
//
// Decode uses the exact per-code tables x_norm(code) of fireflyoptim.py:47-48
// and :77-78 (computed once on the host), replicated 16 times in shared memory
// (entry e of replica k at word e*16+k; lanes l and l+16 share a replica).
// Encode evaluates the mu-law curve as 127/8*log2(1+255|x|) (signed) and
// 255/8*log2(1+255 x) (unsigned): ln(1+255x)/ln(256) = log2(1+255x)/8.
//
// The kernel is bound by instruction issue as much as by HBM, so the fp32 math
// uses the special-function unit's approximations (rsqrt, lg2, tanh) and the
// 1.5*2^23 magic add for rounding and int<->float, each checked against the exact
// formulation where a result could land on a decision boundary: the eps term of
// the Adam denominator, and the stochastic-rounding comparison (an accurate tanh
// is recomputed when |u - threshold| < 2e-4).
#pragma once
#include "ff_common.cuh"

namespace ff {
namespace optim {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kBlock = 256;
constexpr int kRep = 16;                  // table replicas: lanes l and l+16 share one
constexpr int kTabWords = 256 * kRep;     // one replicated table
constexpr int kSmemBytes = 2 * kTabWords * 4;
constexpr float kMagic = 12582912.0f;     // 1.5 * 2^23

struct Params {
  int8_t* q;
  const float* wscale;
  int64_t row_len;
  int64_t elem_base;
  const uint16_t* g;
  uint8_t* m_q;
  float* m_absmax;
  uint8_t* v_q;
  float* v_absmax;
  uint8_t* r_q;
  float* r_absmax;
  int64_t numel;
  float neg_lr, beta1, beta2, eps, wd, sr_bias;
  float omb1, omb2, ibc1, ibc2, bc1, bc2;
  uint32_t seed_lo, seed_hi, step_lo, step_hi;
  int64_t rng_offset;
  int64_t row_step, in_row_step;  // grid-stride advance in (rows, elements within a row)
  const float* u;
  const float* dec_s;
  const float* dec_u;
};

// Philox4x32-10 (Salmon et al., "Parallel random numbers: as easy as 1, 2, 3", SC'11)
__device__ __forceinline__ void philox4x32_10(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, uint32_t k0,
                                              uint32_t k1, uint32_t (&out)[4]) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(0xD2511F53u, c0), lo0 = 0xD2511F53u * c0;
    const uint32_t hi1 = __umulhi(0xCD9E8D57u, c2), lo1 = 0xCD9E8D57u * c2;
    const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
    c0 = n0;
    c1 = lo1;
    c2 = n2;
    c3 = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  out[0] = c0;
  out[1] = c1;
  out[2] = c2;
  out[3] = c3;
}

__device__ __forceinline__ float lg2_approx(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rsqrt_approx(float x) {
  float y;
  asm("rsqrt.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// tanh(x) = 1 - 2 / (1 + e^{2x}), absolute error about 1e-7
__device__ __forceinline__ float tanh_accurate(float x) {
  const float e = ex2_approx(__fmul_rn(x, 2.8853900817779268f));  // 2 / ln 2
  return __fsub_rn(1.f, __fmul_rn(2.f, rcp_approx(__fadd_rn(1.f, e))));
}

// x / d from inv_d ~ 1/d with one residual correction: q0 = x*inv_d, r = x - q0*d (exact by
// FMA), q = q0 + r*inv_d.  This is the correctly rounded quotient except when it lies
// extremely close to a rounding midpoint.
__device__ __forceinline__ float div_nr(float x, float d, float inv_d) {
  const float q0 = __fmul_rn(x, inv_d);
  const float r = __fmaf_rn(-q0, d, x);
  return __fmaf_rn(r, inv_d, q0);
}

// sqrt(x) from rsqrt.approx with one residual correction (x >= 0; x == 0 gives 0)
__device__ __forceinline__ float sqrt_nr(float x) {
  const float rs = rsqrt_approx(x);
  const float s0 = x == 0.f ? 0.f : __fmul_rn(x, rs);
  const float e = __fmaf_rn(-s0, s0, x);
  return x == 0.f ? 0.f : __fmaf_rn(e, __fmul_rn(0.5f, rs), s0);
}

// exact int <-> float for small integers on the FMA/ALU pipes
__device__ __forceinline__ float small_int_to_float(int i) { return __fsub_rn(__int_as_float(0x4B400000 + i), kMagic); }
__device__ __forceinline__ int rne_int(float x) { return __float_as_int(__fadd_rn(x, kMagic)) - 0x4B400000; }

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ uint32_t pack_codes(const int (&c)[8], int base) {
  return (uint32_t)(c[base] & 0xff) | ((uint32_t)(c[base + 1] & 0xff) << 8) |
         ((uint32_t)(c[base + 2] & 0xff) << 16) | ((uint32_t)(c[base + 3] & 0xff) << 24);
}

template <bool HAS_U, bool SMALL_ROWS>
__global__ void __launch_bounds__(kThreads, 3) dqt_adamw8_kernel(Params p) {
  extern __shared__ float tab[];  // [2][256 codes][kRep]
  float* tabS = tab;
  float* tabU = tab + kTabWords;
  for (int i = threadIdx.x; i < kTabWords; i += kThreads) {
    tabS[i] = __ldg(p.dec_s + i / kRep);
    tabU[i] = __ldg(p.dec_u + i / kRep);
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int slot = lane & (kRep - 1);
  const int64_t nblocks = (p.numel + kBlock - 1) / kBlock;
  const int64_t wstride = (int64_t)gridDim.x * kWarps;
  const float eps = p.eps;
  const int64_t last_row = (p.elem_base + p.numel - 1) / p.row_len;
  int64_t blk = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  // weight row of this lane's first element, advanced incrementally (no division per block)
  int64_t row, in_row;
  {
    const int64_t ge = p.elem_base + blk * kBlock + lane * 8;
    row = ge / p.row_len;
    in_row = ge - row * p.row_len;
  }
  for (; blk < nblocks; blk += wstride) {
    const int64_t e0 = blk * kBlock + lane * 8;
    const int nvalid = (int)max64(0, min64(8, p.numel - e0));
    float g[8];
    int qv[8], mc[8], vc[8], rc[8];
    if (nvalid == 8) {
      const uint4 gw = __ldg(reinterpret_cast<const uint4*>(p.g + e0));
      const uint2 qw = *reinterpret_cast<const uint2*>(p.q + e0);
      const uint2 mw = *reinterpret_cast<const uint2*>(p.m_q + e0);
      const uint2 vw = *reinterpret_cast<const uint2*>(p.v_q + e0);
      const uint2 rw = *reinterpret_cast<const uint2*>(p.r_q + e0);
      const uint32_t gws[4] = {gw.x, gw.y, gw.z, gw.w};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        g[j] = __uint_as_float((j & 1) ? (gws[j >> 1] & 0xFFFF0000u) : (gws[j >> 1] << 16));
        const int sh = (j & 3) * 8;
        const uint32_t qwj = j < 4 ? qw.x : qw.y, mwj = j < 4 ? mw.x : mw.y;
        const uint32_t vwj = j < 4 ? vw.x : vw.y, rwj = j < 4 ? rw.x : rw.y;
        qv[j] = (int)(int8_t)((qwj >> sh) & 0xff);
        mc[j] = (int)((mwj >> sh) & 0xff);
        vc[j] = (int)((vwj >> sh) & 0xff);
        rc[j] = (int)((rwj >> sh) & 0xff);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const bool ok = j < nvalid;
        g[j] = ok ? __uint_as_float((uint32_t)p.g[e0 + j] << 16) : 0.f;
        qv[j] = ok ? (int)p.q[e0 + j] : 0;
        mc[j] = ok ? (int)p.m_q[e0 + j] : 128;
        vc[j] = ok ? (int)p.v_q[e0 + j] : 0;
        rc[j] = ok ? (int)p.r_q[e0 + j] : 128;
      }
    }
    const float am = __ldg(p.m_absmax + blk), av = __ldg(p.v_absmax + blk), ar = __ldg(p.r_absmax + blk);
    float u[8];
    if constexpr (HAS_U) {
#pragma unroll
      for (int j = 0; j < 8; ++j) u[j] = j < nvalid ? __ldg(p.u + e0 + j) : 2.f;
    } else {
      uint32_t w[4];
      const uint64_t call = (uint64_t)(p.rng_offset + e0) >> 3;
      philox4x32_10((uint32_t)call, (uint32_t)(call >> 32), p.step_lo, p.step_hi, p.seed_lo, p.seed_hi, w);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint32_t h = (j & 1) ? (w[j >> 1] >> 16) : (w[j >> 1] & 0xFFFFu);
        u[j] = __fmul_rn(__fsub_rn(__int_as_float(0x4B000000 | h), 8388608.f) + 0.5f, 1.0f / 65536.0f);
      }
    }
    // weight-row scales: with row_len >= 8 the 8 elements span at most two rows
    const int64_t ra = min64(row, last_row), rb = min64(row + 1, last_row);
    const int jsw = SMALL_ROWS ? 8 : (int)min64(8, p.row_len - in_row);  // j >= jsw: next row
    const float wsa = fmaxf(__ldg(p.wscale + ra), eps);
    const float wsb = jsw < 8 ? fmaxf(__ldg(p.wscale + rb), eps) : wsa;
    const float iwsa = __frcp_rn(wsa), iwsb = __frcp_rn(wsb);
    float mn[8], vn[8], rn[8];
    int qn[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float ws = j < jsw ? wsa : wsb, iws = j < jsw ? iwsa : iwsb;
      if constexpr (SMALL_ROWS) {  // rows shorter than 8 elements: one division per element
        ws = fmaxf(__ldg(p.wscale + min64((p.elem_base + min64(e0 + j, p.numel - 1)) / p.row_len, last_row)), eps);
        iws = __frcp_rn(ws);
      }
      float m = __fmul_rn(tabS[mc[j] * kRep + slot], am);
      float v = __fmul_rn(tabU[vc[j] * kRep + slot], av);
      float r = __fmul_rn(tabS[rc[j] * kRep + slot], ar);
      const float gj = g[j];
      m = __fmaf_rn(gj, p.omb1, __fmul_rn(m, p.beta1));
      v = __fmaf_rn(__fmul_rn(p.omb2, gj), gj, __fmul_rn(v, p.beta2));
      // the residual update below loses its leading digits when dq is subtracted, so
      // this chain follows the reference's rounding step by step (fireflyoptim.py:177-184)
      const float mh = div_nr(m, p.bc1, p.ibc1);
      const float vh = div_nr(v, p.bc2, p.ibc2);
      const float den = __fadd_rn(sqrt_nr(vh), eps);
      const float a = div_nr(mh, den, rcp_approx(den));
      const float qf = small_int_to_float(qv[j]);
      const float dwe = __fmul_rn(p.neg_lr, __fadd_rn(a, __fmul_rn(__fmul_rn(p.wd, qf), ws)));
      r = __fadd_rn(r, div_nr(dwe, ws, iws));
      const float absr = fabsf(r);
      float base;
      if (absr < 4194304.f) {  // floor via the magic add (exact below 2^22)
        base = __fsub_rn(__fadd_rn(__fsub_rn(absr, 0.5f), kMagic), kMagic);
        if (__fadd_rn(base, 1.f) <= absr) base = __fadd_rn(base, 1.f);
      } else {
        base = floorf(absr);
      }
      const float frac = __fsub_rn(absr, base);
      const float sgn = r > 0.f ? 1.f : (r < 0.f ? -1.f : 0.f);
      float fb = frac;
      if (p.sr_bias != 0.f) {
        fb = __fadd_rn(frac, __fmul_rn(__fmul_rn(tanh_approx(a), p.sr_bias), sgn));
        // tanh.approx is good to ~5e-4: near the decision use an accurate tanh
        if (fabsf(__fsub_rn(u[j], fb)) < 2e-4f)
          fb = __fadd_rn(frac, __fmul_rn(__fmul_rn(tanh_accurate(a), p.sr_bias), sgn));
      }
      fb = fminf(fmaxf(fb, 0.f), 1.f);
      const float extra = (u[j] < fb) ? 1.f : 0.f;
      const float dqf = fminf(fmaxf(__fmul_rn(sgn, __fadd_rn(base, extra)), -2097152.f), 2097152.f);
      if (j < nvalid) {
        qn[j] = max(-127, min(127, qv[j] + rne_int(dqf)));
        r = __fsub_rn(r, dqf);
      } else {
        qn[j] = 0;
        r = 0.f;
        m = 0.f;
        v = 0.f;
      }
      mn[j] = m;
      vn[j] = v;
      rn[j] = r;
    }
    // ---------------- block absmax and re-encode (mu-law, fireflyoptim.py:22-67)
    float xm = 0.f, xv = 0.f, xr = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      xm = fmaxf(xm, fabsf(mn[j]));
      xv = fmaxf(xv, vn[j]);
      xr = fmaxf(xr, fabsf(rn[j]));
    }
    xm = fmaxf(warp_max(xm), 1e-12f);
    xv = fmaxf(warp_max(xv), 1e-12f);
    xr = fmaxf(warp_max(xr), 1e-12f);
    const float ixm = __frcp_rn(xm), ixv = __frcp_rn(xv), ixr = __frcp_rn(xr);
    int cm[8], cv[8], cr[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float nm = fminf(fabsf(__fmul_rn(mn[j], ixm)), 1.f);
      const float nr = fminf(fabsf(__fmul_rn(rn[j], ixr)), 1.f);
      const float nv = fminf(fmaxf(__fmul_rn(vn[j], ixv), 0.f), 1.f);
      const float lm = __fmul_rn(lg2_approx(__fmaf_rn(255.f, nm, 1.f)), 15.875f);
      const float lr = __fmul_rn(lg2_approx(__fmaf_rn(255.f, nr, 1.f)), 15.875f);
      const float lv = __fmul_rn(lg2_approx(__fmaf_rn(255.f, nv, 1.f)), 31.875f);
      cm[j] = min(255, max(1, rne_int(__fadd_rn(copysignf(lm, mn[j]), 128.f))));
      cr[j] = min(255, max(1, rne_int(__fadd_rn(copysignf(lr, rn[j]), 128.f))));
      cv[j] = min(255, max(0, rne_int(lv)));
    }
    if (nvalid == 8) {
      *reinterpret_cast<uint2*>(p.q + e0) = make_uint2(pack_codes(qn, 0), pack_codes(qn, 4));
      *reinterpret_cast<uint2*>(p.m_q + e0) = make_uint2(pack_codes(cm, 0), pack_codes(cm, 4));
      *reinterpret_cast<uint2*>(p.v_q + e0) = make_uint2(pack_codes(cv, 0), pack_codes(cv, 4));
      *reinterpret_cast<uint2*>(p.r_q + e0) = make_uint2(pack_codes(cr, 0), pack_codes(cr, 4));
    } else {
      for (int j = 0; j < nvalid; ++j) {
        p.q[e0 + j] = (int8_t)qn[j];
        p.m_q[e0 + j] = (uint8_t)cm[j];
        p.v_q[e0 + j] = (uint8_t)cv[j];
        p.r_q[e0 + j] = (uint8_t)cr[j];
      }
    }
    if (lane == 0) {
      p.m_absmax[blk] = xm;
      p.v_absmax[blk] = xv;
      p.r_absmax[blk] = xr;
    }
    row += p.row_step;
    in_row += p.in_row_step;
    if (in_row >= p.row_len) {
      in_row -= p.row_len;
      ++row;
    }
  }
}

}  // namespace optim
}  // namespace ff

extern "C" int ff_dqt_adamw8(int8_t* q, const float* wscale, int64_t row_len, int64_t elem_base, const uint16_t* g,
                             uint8_t* m_q, float* m_absmax, uint8_t* v_q, float* v_absmax, uint8_t* r_q,
                             float* r_absmax, int64_t numel, int64_t block, double lr, double beta1,
                             double beta2, double eps, double wd, double bc1, double bc2, double sr_bias,
                             uint64_t seed, uint64_t step,
                             int64_t rng_offset, const float* u, const float* dec_s, const float* dec_u,
                             void* stream) {
  using namespace ff;
  using namespace ff::optim;
  FF_REQUIRE(numel >= 0 && row_len >= 1 && elem_base >= 0 && rng_offset >= 0, FF_ERR_INVALID_ARG,
             "ff_dqt_adamw8: bad sizes");
  FF_REQUIRE(block == kBlock, FF_ERR_UNSUPPORTED, "ff_dqt_adamw8: block must be %d (got %lld)", kBlock,
             (long long)block);
  if (numel == 0) return FF_OK;
  FF_REQUIRE(q && wscale && g && m_q && m_absmax && v_q && v_absmax && r_q && r_absmax && dec_s && dec_u,
             FF_ERR_INVALID_ARG, "ff_dqt_adamw8: null pointer");
  FF_REQUIRE(aligned(g, 16) && aligned(q, 8) && aligned(m_q, 8) && aligned(v_q, 8) && aligned(r_q, 8),
             FF_ERR_UNSUPPORTED, "ff_dqt_adamw8: g needs 16-byte and code arrays 8-byte alignment");
  FF_REQUIRE(rng_offset % 8 == 0, FF_ERR_UNSUPPORTED, "ff_dqt_adamw8: rng_offset must be a multiple of 8");
  FF_REQUIRE(bc1 > 0.0 && bc2 > 0.0, FF_ERR_INVALID_ARG, "ff_dqt_adamw8: bias corrections must be > 0");
  Params p;
  p.q = q;
  p.wscale = wscale;
  p.row_len = row_len;
  p.elem_base = elem_base;
  p.g = g;
  p.m_q = m_q;
  p.m_absmax = m_absmax;
  p.v_q = v_q;
  p.v_absmax = v_absmax;
  p.r_q = r_q;
  p.r_absmax = r_absmax;
  p.numel = numel;
  // scalars are rounded to fp32 the way torch does for a python float operand
  p.neg_lr = (float)(-lr);
  p.beta1 = (float)beta1;
  p.beta2 = (float)beta2;
  p.eps = (float)eps;
  p.wd = (float)wd;
  p.sr_bias = (float)sr_bias;
  p.omb1 = (float)(1.0 - beta1);
  p.omb2 = (float)(1.0 - beta2);
  p.bc1 = (float)bc1;
  p.bc2 = (float)bc2;
  p.ibc1 = (float)(1.0 / (double)p.bc1);
  p.ibc2 = (float)(1.0 / (double)p.bc2);
  p.seed_lo = (uint32_t)seed;
  p.seed_hi = (uint32_t)(seed >> 32);
  p.step_lo = (uint32_t)step;
  p.step_hi = (uint32_t)(step >> 32);
  p.rng_offset = rng_offset;
  p.u = u;
  p.dec_s = dec_s;
  p.dec_u = dec_u;
  int dev = 0;
  cudaGetDevice(&dev);
  static bool attr_set[64] = {false};
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    FF_CUDA_TRY(cudaFuncSetAttribute(dqt_adamw8_kernel<true, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemBytes), "ff_dqt_adamw8 smem attribute");
    FF_CUDA_TRY(cudaFuncSetAttribute(dqt_adamw8_kernel<false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemBytes), "ff_dqt_adamw8 smem attribute");
    FF_CUDA_TRY(cudaFuncSetAttribute(dqt_adamw8_kernel<true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemBytes), "ff_dqt_adamw8 smem attribute");
    FF_CUDA_TRY(cudaFuncSetAttribute(dqt_adamw8_kernel<false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemBytes), "ff_dqt_adamw8 smem attribute");
    attr_set[dev] = true;
  }
  const int64_t nblocks = (numel + kBlock - 1) / kBlock;
  int nsm = 148;
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (nblocks + kWarps - 1) / kWarps;
  const int grid = (int)min64(want, (int64_t)nsm * 3);
  const int64_t stride_elems = (int64_t)grid * kWarps * kBlock;
  p.row_step = stride_elems / row_len;
  p.in_row_step = stride_elems % row_len;
  cudaStream_t st = as_stream(stream);
  const bool small = row_len < 8;
  if (u) {
    if (small) dqt_adamw8_kernel<true, true><<<grid, kThreads, kSmemBytes, st>>>(p);
    else dqt_adamw8_kernel<true, false><<<grid, kThreads, kSmemBytes, st>>>(p);
  } else {
    if (small) dqt_adamw8_kernel<false, true><<<grid, kThreads, kSmemBytes, st>>>(p);
    else dqt_adamw8_kernel<false, false><<<grid, kThreads, kSmemBytes, st>>>(p);
  }
  return check_launch("ff_dqt_adamw8");
}
