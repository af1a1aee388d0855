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
constexpr int kTabBytes = 2 * kTabWords * 4;
// per warp, two stages of one block's inputs, filled by 1-D bulk (TMA) copies:
// g (512 B) | q (256) | m (256) | v (256) | r (256) | u (1024, parity mode only)
constexpr int kStageBytes = 512 + 4 * 256 + 1024;
constexpr int kStageOffQ = 512, kStageOffM = 768, kStageOffV = 1024, kStageOffR = 1280, kStageOffU = 1536;
constexpr int kSmemBytes = kTabBytes + kWarps * 2 * kStageBytes + kWarps * 2 * 8;
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
  int bulk;                       // all arrays 16-byte aligned: stage inputs with bulk copies
  const float* u;
  const float* dec_s;
  const float* dec_u;
};

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void bar_init(uint32_t bar) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar));
}
__device__ __forceinline__ void bar_expect(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool bar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// time-bounded wait; false (and FF_DEVICE_TIMEOUT raised) if the copies never landed
__device__ __forceinline__ bool bar_wait(uint32_t bar, uint32_t parity) {
  if (bar_try(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (!bar_try(bar, parity)) {
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      raise_status(FF_DEVICE_TIMEOUT);
      return false;
    }
  }
  return true;
}
// 1-D bulk copy global -> shared (no multicast), completion counted on `bar`
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

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

// sqrt(x) from rsqrt.approx with one residual correction, x >= 0.  Arguments below
// 1e-37 (whose square roots are far below any eps added to them) use rsqrt(1e-37), so
// x == 0 gives exactly 0 without a select.
__device__ __forceinline__ float sqrt_nr(float x) {
  const float rs = rsqrt_approx(fmaxf(x, 1e-37f));
  const float s0 = __fmul_rn(x, rs);
  const float e = __fmaf_rn(-s0, s0, x);
  return __fmaf_rn(e, __fmul_rn(0.5f, rs), s0);
}

// exact int <-> float for small integers on the FMA/ALU pipes
__device__ __forceinline__ float small_int_to_float(int i) { return __fsub_rn(__int_as_float(0x4B400000 + i), kMagic); }
__device__ __forceinline__ int rne_int(float x) { return __float_as_int(__fadd_rn(x, kMagic)) - 0x4B400000; }

// maximum over the warp of non-negative floats: their bit patterns order like the values,
// so one integer reduction does it
__device__ __forceinline__ float warp_max_nonneg(float v) {
  return __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(v)));
}

// low bytes of four ints -> one word (byte permutes)
__device__ __forceinline__ uint32_t pack_codes(const int (&c)[8], int base) {
  const uint32_t lo = __byte_perm((uint32_t)c[base], (uint32_t)c[base + 1], 0x0040);
  const uint32_t hi = __byte_perm((uint32_t)c[base + 2], (uint32_t)c[base + 3], 0x0040);
  return __byte_perm(lo, hi, 0x5410);
}

// x / d with nd = -d and id ~ 1/d: q0 = x*id, r = x - q0*d (exact), q = q0 + r*id
__device__ __forceinline__ f2 div2(f2 x, f2 nd, f2 id) {
  const f2 q0 = mul2(x, id);
  return fma2(fma2(q0, nd, x), id, q0);
}

__device__ __forceinline__ uint32_t byte_of(uint32_t w, int k) { return (w >> (8 * k)) & 0xFFu; }

// ROWS: 0 = row_len a multiple of 8 (a lane's 8 elements share one weight row),
//       1 = row_len >= 8 (they span at most two rows), 2 = row_len < 8
template <bool HAS_U, int ROWS>
__global__ void __launch_bounds__(kThreads, 3) dqt_adamw8_kernel(Params p) {
  extern __shared__ __align__(128) float tab[];  // [2][256 codes][kRep], then staging, then barriers
  float* tabS = tab;
  float* tabU = tab + kTabWords;
  uint8_t* stage_base = reinterpret_cast<uint8_t*>(tab) + kTabBytes;
  const int warp = threadIdx.x >> 5;
  uint8_t* my_stage = stage_base + warp * 2 * kStageBytes;
  const uint32_t bar0 = smem_addr(stage_base + kWarps * 2 * kStageBytes) + warp * 16;
  for (int i = threadIdx.x; i < kTabWords; i += kThreads) {
    tabS[i] = __ldg(p.dec_s + i / kRep);
    tabU[i] = __ldg(p.dec_u + i / kRep);
  }
  if ((threadIdx.x & 31) == 0) {
    bar_init(bar0);
    bar_init(bar0 + 8);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int slot = lane & (kRep - 1);
  const uint32_t stage_bytes_tx = 512 + 4 * 256 + (HAS_U ? 1024 : 0);
  // lane 0 stages block b (a full block) into stage s
  auto prefetch = [&](int64_t b, int s) {
    const uint32_t dst = smem_addr(my_stage + s * kStageBytes), bar = bar0 + 8 * s;
    const int64_t e = b * kBlock;
    bar_expect(bar, stage_bytes_tx);
    bulk_g2s(dst, p.g + e, 512, bar);
    bulk_g2s(dst + kStageOffQ, p.q + e, 256, bar);
    bulk_g2s(dst + kStageOffM, p.m_q + e, 256, bar);
    bulk_g2s(dst + kStageOffV, p.v_q + e, 256, bar);
    bulk_g2s(dst + kStageOffR, p.r_q + e, 256, bar);
    if constexpr (HAS_U) bulk_g2s(dst + kStageOffU, p.u + e, 1024, bar);
  };
  const int64_t full_blocks = p.numel / kBlock;  // blocks [0, full_blocks) have 256 elements
  const int64_t nblocks = (p.numel + kBlock - 1) / kBlock;
  const int64_t wstride = (int64_t)gridDim.x * kWarps;
  const float eps = p.eps;
  const int64_t last_row = (p.elem_base + p.numel - 1) / p.row_len;
  // loop-invariant pairs
  const f2 b1 = splat(p.beta1), b2 = splat(p.beta2), omb1 = splat(p.omb1), omb2 = splat(p.omb2);
  const f2 nbc1 = splat(-p.bc1), nbc2 = splat(-p.bc2), ibc1 = splat(p.ibc1), ibc2 = splat(p.ibc2);
  const f2 eps2 = splat(eps), nlr = splat(p.neg_lr), wd2 = splat(p.wd), magic2 = splat(kMagic);
  const f2 half2 = splat(0.5f), mone2 = splat(-1.f);
  int64_t blk = (int64_t)blockIdx.x * kWarps + warp;
  // weight row of this lane's first element, advanced incrementally (no division per block)
  int64_t row, in_row;
  {
    const int64_t ge = p.elem_base + blk * kBlock + lane * 8;
    row = ge / p.row_len;
    in_row = ge - row * p.row_len;
  }
  if (p.bulk && lane == 0 && blk < full_blocks) prefetch(blk, 0);
  for (int it = 0; blk < nblocks; blk += wstride, ++it) {
    const int64_t e0 = blk * kBlock + lane * 8;
    const int nvalid = (int)max64(0, min64(8, p.numel - e0));
    const int stg = it & 1;
    const bool staged = p.bulk && blk < full_blocks;
    // stage the next block while this one is computed (its stage was consumed last iteration)
    if (p.bulk && lane == 0 && blk + wstride < full_blocks) prefetch(blk + wstride, stg ^ 1);
    const float am = __ldg(p.m_absmax + blk), av = __ldg(p.v_absmax + blk), ar = __ldg(p.r_absmax + blk);
    // ---------------- inputs as packed words: g (bf16 pairs), q/m/v/r (bytes)
    uint32_t gw[4], qw[2], mw[2], vw[2], rw[2];
    float u[HAS_U ? 8 : 1];
    if (staged) {
      if (!bar_wait(bar0 + 8 * stg, (it >> 1) & 1)) return;  // copies lost: status raised
      const uint8_t* sb = my_stage + stg * kStageBytes;
      const uint4 g4 = *reinterpret_cast<const uint4*>(sb + lane * 16);
      const uint2 q2 = *reinterpret_cast<const uint2*>(sb + kStageOffQ + lane * 8);
      const uint2 m2 = *reinterpret_cast<const uint2*>(sb + kStageOffM + lane * 8);
      const uint2 v2 = *reinterpret_cast<const uint2*>(sb + kStageOffV + lane * 8);
      const uint2 r2 = *reinterpret_cast<const uint2*>(sb + kStageOffR + lane * 8);
      gw[0] = g4.x; gw[1] = g4.y; gw[2] = g4.z; gw[3] = g4.w;
      qw[0] = q2.x; qw[1] = q2.y; mw[0] = m2.x; mw[1] = m2.y;
      vw[0] = v2.x; vw[1] = v2.y; rw[0] = r2.x; rw[1] = r2.y;
      if constexpr (HAS_U) {
        const float4 u0 = *reinterpret_cast<const float4*>(sb + kStageOffU + lane * 32);
        const float4 u1 = *reinterpret_cast<const float4*>(sb + kStageOffU + lane * 32 + 16);
        u[0] = u0.x; u[1] = u0.y; u[2] = u0.z; u[3] = u0.w;
        u[4] = u1.x; u[5] = u1.y; u[6] = u1.z; u[7] = u1.w;
      }
      __syncwarp();  // every lane has its inputs: the stage may be refilled next iteration
    } else if (nvalid == 8) {
      const uint4 g4 = __ldg(reinterpret_cast<const uint4*>(p.g + e0));
      const uint2 q2 = *reinterpret_cast<const uint2*>(p.q + e0);
      const uint2 m2 = *reinterpret_cast<const uint2*>(p.m_q + e0);
      const uint2 v2 = *reinterpret_cast<const uint2*>(p.v_q + e0);
      const uint2 r2 = *reinterpret_cast<const uint2*>(p.r_q + e0);
      gw[0] = g4.x; gw[1] = g4.y; gw[2] = g4.z; gw[3] = g4.w;
      qw[0] = q2.x; qw[1] = q2.y; mw[0] = m2.x; mw[1] = m2.y;
      vw[0] = v2.x; vw[1] = v2.y; rw[0] = r2.x; rw[1] = r2.y;
      if constexpr (HAS_U) {
#pragma unroll
        for (int j = 0; j < 8; ++j) u[j] = __ldg(p.u + e0 + j);
      }
    } else {
      // ragged tail of the last block: missing elements get g = 0, q = 0 and the zero
      // codes (m, r: 128; v: 0), which the update maps to zeros (ignored by the absmax)
      gw[0] = gw[1] = gw[2] = gw[3] = 0u;
      qw[0] = qw[1] = 0u;
      mw[0] = mw[1] = rw[0] = rw[1] = 0x80808080u;
      vw[0] = vw[1] = 0u;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (j < nvalid) {
          const int sh = 8 * (j & 3), w = j >> 2;
          gw[j >> 1] |= (uint32_t)p.g[e0 + j] << (16 * (j & 1));
          qw[w] |= ((uint32_t)(uint8_t)p.q[e0 + j]) << sh;
          mw[w] = (mw[w] & ~(0xFFu << sh)) | ((uint32_t)p.m_q[e0 + j] << sh);
          vw[w] |= (uint32_t)p.v_q[e0 + j] << sh;
          rw[w] = (rw[w] & ~(0xFFu << sh)) | ((uint32_t)p.r_q[e0 + j] << sh);
        }
        if constexpr (HAS_U) u[j] = j < nvalid ? __ldg(p.u + e0 + j) : 2.f;
      }
    }
    uint32_t rw4[4];  // Philox output: 16 bits per element
    if constexpr (!HAS_U) {
      const uint64_t call = (uint64_t)(p.rng_offset + e0) >> 3;
      philox4x32_10((uint32_t)call, (uint32_t)(call >> 32), p.step_lo, p.step_hi, p.seed_lo, p.seed_hi, rw4);
    }
    // weight-row scales: with row_len >= 8 the 8 elements span at most two rows
    const int64_t ra = min64(row, last_row), rb = min64(row + 1, last_row);
    const int jsw = ROWS != 1 ? 8 : (int)min64(8, p.row_len - in_row);  // j >= jsw: next row
    const float wsa = fmaxf(__ldg(p.wscale + ra), eps);
    const float wsb = jsw < 8 ? fmaxf(__ldg(p.wscale + rb), eps) : wsa;
    const float iwsa = __frcp_rn(wsa), iwsb = __frcp_rn(wsb);
    const f2 am2 = splat(am), av2 = splat(av), ar2 = splat(ar);
    f2 mn[4], vn[4], rn[4];
    int qn[8];
#pragma unroll
    for (int pp = 0; pp < 4; ++pp) {
      const int j0 = 2 * pp, j1 = 2 * pp + 1;
      const int w = pp >> 1, k0 = j0 & 3, k1 = j1 & 3;
      // weight-row scale of both elements
      float ws0 = j0 < jsw ? wsa : wsb, ws1 = j1 < jsw ? wsa : wsb;
      float iws0 = j0 < jsw ? iwsa : iwsb, iws1 = j1 < jsw ? iwsa : iwsb;
      if constexpr (ROWS == 2) {  // rows shorter than 8 elements: one division per element
        ws0 = fmaxf(__ldg(p.wscale + min64((p.elem_base + min64(e0 + j0, p.numel - 1)) / p.row_len, last_row)), eps);
        ws1 = fmaxf(__ldg(p.wscale + min64((p.elem_base + min64(e0 + j1, p.numel - 1)) / p.row_len, last_row)), eps);
        iws0 = __frcp_rn(ws0);
        iws1 = __frcp_rn(ws1);
      }
      const f2 ws = mk2(ws0, ws1), nws = mk2(-ws0, -ws1), iws = mk2(iws0, iws1);
      // decode (fireflyoptim.py:39-80): table value * block absmax
      const f2 g = mk2(__uint_as_float(gw[pp] << 16), __uint_as_float(gw[pp] & 0xFFFF0000u));
      f2 m = mul2(mk2(tabS[byte_of(mw[w], k0) * kRep + slot], tabS[byte_of(mw[w], k1) * kRep + slot]), am2);
      f2 v = mul2(mk2(tabU[byte_of(vw[w], k0) * kRep + slot], tabU[byte_of(vw[w], k1) * kRep + slot]), av2);
      f2 r = mul2(mk2(tabS[byte_of(rw[w], k0) * kRep + slot], tabS[byte_of(rw[w], k1) * kRep + slot]), ar2);
      // Adam moments (fireflyoptim.py:175-178); the chain below follows the reference's
      // rounding step by step because the residual loses its leading digits when dq is
      // subtracted (fireflyoptim.py:177-184)
      m = fma2(g, omb1, mul2(m, b1));
      v = fma2(mul2(omb2, g), g, mul2(v, b2));
      const f2 mh = div2(m, nbc1, ibc1);
      const f2 vh = div2(v, nbc2, ibc2);
      float vh0, vh1;
      un2(vh, vh0, vh1);
      // sqrt from rsqrt.approx with one residual correction; arguments below 1e-37 (square
      // roots far below eps) use rsqrt(1e-37) so that sqrt(0) = 0 exactly
      const f2 rs = mk2(rsqrt_approx(fmaxf(vh0, 1e-37f)), rsqrt_approx(fmaxf(vh1, 1e-37f)));
      const f2 s0 = mul2(vh, rs);
      const f2 sq = fma2(fma2(s0, mul2(s0, mone2), vh), mul2(rs, half2), s0);
      const f2 den = add2(sq, eps2);
      float d0, d1;
      un2(den, d0, d1);
      const f2 a = div2(mh, mul2(den, mone2), mk2(rcp_approx(d0), rcp_approx(d1)));
      // DQT residual (fireflyoptim.py:180-184)
      const int q0 = (int)(int8_t)byte_of(qw[w], k0), q1 = (int)(int8_t)byte_of(qw[w], k1);
      const f2 qf = sub2(mk2(__int_as_float(0x4B400000 + q0), __int_as_float(0x4B400000 + q1)), magic2);
      const f2 dwe = mul2(nlr, add2(a, mul2(mul2(wd2, qf), ws)));
      r = add2(r, div2(dwe, nws, iws));
      // momentum-biased stochastic rounding (fireflyoptim.py:186-198)
      float r0, r1, a0, a1;
      un2(r, r0, r1);
      un2(a, a0, a1);
      // |r| is clamped to 2^21 (far above any reachable residual) so that the floor and the
      // integer conversion below are exact magic-number adds
      const f2 absr = mk2(fminf(fabsf(r0), 2097152.f), fminf(fabsf(r1), 2097152.f));
      const f2 base = sub2(add2_rm(absr, magic2), magic2);  // floor(|r|)
      const f2 frac = sub2(absr, base);
      float fr0, fr1, bs0, bs1;
      un2(frac, fr0, fr1);
      un2(base, bs0, bs1);
      float uj[2];
      if constexpr (HAS_U) {
        uj[0] = u[j0];
        uj[1] = u[j1];
      } else {
        // u = (h + 0.5) / 65536 for the 16-bit halves h of the Philox word: 2^23 + h is built by a
        // byte permute, and (2^23 + h) * 2^-16 + (2^-17 - 128) is exact in one FMA
        const uint32_t wd_ = rw4[pp];
        un2(fma2(mk2(__int_as_float(__byte_perm(wd_, 0x4B000000u, 0x7610)),
                     __int_as_float(__byte_perm(wd_, 0x4B000000u, 0x7632))),
                 splat(1.0f / 65536.0f), splat(1.0f / 131072.0f - 128.0f)),
            uj[0], uj[1]);
      }
      const float rr[2] = {r0, r1}, aa[2] = {a0, a1}, fr[2] = {fr0, fr1}, bs[2] = {bs0, bs1};
      float dqf[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        // threshold frac(|r|) + tanh(a) * sr_bias * sign(r); tb * sign(r) is tb with its sign
        // flipped for negative r (r = 0 is handled below: dq = sign(0) * ... = 0)
        const uint32_t rsign = __float_as_uint(rr[e]) & 0x80000000u;
        float fb = fr[e];
        if (p.sr_bias != 0.f) {
          const float tb = __fmul_rn(tanh_approx(aa[e]), p.sr_bias);
          fb = __fadd_rn(fr[e], __uint_as_float(__float_as_uint(tb) ^ rsign));
          // tanh.approx is good to ~5e-4: near the decision use an accurate tanh
          if (fabsf(__fsub_rn(uj[e], fb)) < 2e-4f) {
            const float tb2 = __fmul_rn(tanh_accurate(aa[e]), p.sr_bias);
            fb = __fadd_rn(fr[e], __uint_as_float(__float_as_uint(tb2) ^ rsign));
          }
        }
        // u in (0,1): u < fb is u < clamp(fb, 0, 1); dq = sign(r) * (floor|r| + [u < fb])
        const bool up = (uj[e] < fb) && (rr[e] != 0.f);
        dqf[e] = copysignf(up ? __fadd_rn(bs[e], 1.f) : bs[e], rr[e]);
      }
      qn[j0] = max(-127, min(127, q0 + rne_int(dqf[0])));
      qn[j1] = max(-127, min(127, q1 + rne_int(dqf[1])));
      rn[pp] = sub2(r, mk2(dqf[0], dqf[1]));
      mn[pp] = m;
      vn[pp] = v;
    }
    // ---------------- block absmax and re-encode (mu-law, fireflyoptim.py:22-67)
    float xm = 0.f, xv = 0.f, xr = 0.f;
#pragma unroll
    for (int pp = 0; pp < 4; ++pp) {
      float a0, a1;
      un2(mn[pp], a0, a1);
      xm = fmaxf(xm, fmaxf(fabsf(a0), fabsf(a1)));
      un2(vn[pp], a0, a1);
      xv = fmaxf(xv, fmaxf(fabsf(a0), fabsf(a1)));  // v >= 0; |.| turns -0 into +0
      un2(rn[pp], a0, a1);
      xr = fmaxf(xr, fmaxf(fabsf(a0), fabsf(a1)));
    }
    xm = fmaxf(warp_max_nonneg(xm), 1e-12f);
    xv = fmaxf(warp_max_nonneg(xv), 1e-12f);
    xr = fmaxf(warp_max_nonneg(xr), 1e-12f);
    const f2 ixm = splat(__frcp_rn(xm)), ixv = splat(__frcp_rn(xv)), ixr = splat(__frcp_rn(xr));
    const f2 k127 = splat(15.875f), k255 = splat(31.875f);
    int cm[8], cv[8], cr[8];
    // |x| / absmax can exceed 1 by an ulp (absmax is the largest |x|); log2(256 + tiny) * 127/8
    // still rounds to 127 (255 for v), so no clamps are needed.  v is never negative.
#pragma unroll
    for (int pp = 0; pp < 4; ++pp) {
      float x0, x1, y0, y1, z0, z1;
      un2(mul2(mn[pp], ixm), x0, x1);
      un2(mul2(rn[pp], ixr), y0, y1);
      un2(mul2(vn[pp], ixv), z0, z1);
      // signed m and r: code = 128 + sign(x) * rint(127/8 * log2(1 + 255 |x|/absmax))
      float lm0, lm1, lr0, lr1, lv0, lv1;
      un2(mul2(mk2(lg2_approx(__fmaf_rn(255.f, fabsf(x0), 1.f)), lg2_approx(__fmaf_rn(255.f, fabsf(x1), 1.f))), k127),
          lm0, lm1);
      un2(mul2(mk2(lg2_approx(__fmaf_rn(255.f, fabsf(y0), 1.f)), lg2_approx(__fmaf_rn(255.f, fabsf(y1), 1.f))), k127),
          lr0, lr1);
      // unsigned v: code = rint(255/8 * log2(1 + 255 v/absmax)), +magic folded in
      un2(fma2(mk2(lg2_approx(__fmaf_rn(255.f, z0, 1.f)), lg2_approx(__fmaf_rn(255.f, z1, 1.f))), k255, magic2),
          lv0, lv1);
      // rounding with +128 folded into the magic add
      float s0, s1;
      // the magic-number words themselves: their low byte is the code (0x4B400000 + c, 0 <= c < 256)
      un2(add2(mk2(copysignf(lm0, x0), copysignf(lm1, x1)), splat(kMagic + 128.f)), s0, s1);
      cm[2 * pp] = __float_as_int(s0);
      cm[2 * pp + 1] = __float_as_int(s1);
      un2(add2(mk2(copysignf(lr0, y0), copysignf(lr1, y1)), splat(kMagic + 128.f)), s0, s1);
      cr[2 * pp] = __float_as_int(s0);
      cr[2 * pp + 1] = __float_as_int(s1);
      cv[2 * pp] = __float_as_int(lv0);
      cv[2 * pp + 1] = __float_as_int(lv1);
    }
    if (nvalid == 8) {
      // generic-proxy stores; the bulk copies only ever read other blocks
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
  p.bulk = aligned(q, 16) && aligned(m_q, 16) && aligned(v_q, 16) && aligned(r_q, 16) && (!u || aligned(u, 16));
  int dev = 0;
  cudaGetDevice(&dev);
  static bool attr_set[64] = {false};
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    const void* fns[] = {(const void*)dqt_adamw8_kernel<true, 0>, (const void*)dqt_adamw8_kernel<true, 1>,
                         (const void*)dqt_adamw8_kernel<true, 2>, (const void*)dqt_adamw8_kernel<false, 0>,
                         (const void*)dqt_adamw8_kernel<false, 1>, (const void*)dqt_adamw8_kernel<false, 2>};
    for (const void* fn : fns)
      FF_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes),
                  "ff_dqt_adamw8 smem attribute");
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
  // a lane's 8 elements start at a multiple of 8 of the weight when elem_base is one
  const int rows_mode = (row_len % 8 == 0 && elem_base % 8 == 0) ? 0 : (row_len >= 8 ? 1 : 2);
#define FF_DQT_LAUNCH(HU, RM) dqt_adamw8_kernel<HU, RM><<<grid, kThreads, kSmemBytes, st>>>(p)
  if (u) {
    if (rows_mode == 0) FF_DQT_LAUNCH(true, 0);
    else if (rows_mode == 1) FF_DQT_LAUNCH(true, 1);
    else FF_DQT_LAUNCH(true, 2);
  } else {
    if (rows_mode == 0) FF_DQT_LAUNCH(false, 0);
    else if (rows_mode == 1) FF_DQT_LAUNCH(false, 1);
    else FF_DQT_LAUNCH(false, 2);
  }
#undef FF_DQT_LAUNCH
  return check_launch("ff_dqt_adamw8");
}
