// ff_dqt_adamw8.cuh — fused DQT-SR 8-bit AdamW update of int8 weights (one HBM pass).
//
// Replaces the per-module body of FireFlyOptim.step (fireflyoptim.py:137-209):
// ~40 torch elementwise passes plus a host sync become one kernel that reads
// g (bf16), q (int8), the m/v/r uint8 codes and their block absmax, and
// writes q, the codes and the new absmax.
//
// Work split: one warp per 256-element block, 8 consecutive elements per lane
// (16 B of g, 8 B of each code array per lane: fully coalesced), staged into
// shared memory by per-warp double-buffered 1-D bulk copies.  The block absmax of
// the re-encoded r, m, v is a warp max-reduction.
//
// The kernel is bound by instruction issue (about 10 B of HBM traffic per element
// against some 60 instructions), so every step is written for the fewest issue slots:
//
// * Decode.  The decode tables x_norm(code) of fireflyoptim.py:47-48 and :77-78
//   (computed on the host by the reference formula) sit in shared memory as 256
//   rows of 256 bytes: row c holds 32 copies of the signed entry (one per lane)
//   and 32 of the unsigned one.  The byte offset of lane l's copy of code c is
//   c*256 + 4*l, which one byte permute builds from the code word and the lane's
//   4*l: a decode is one permute and one conflict-free shared load.
// * Packed pairs.  Two elements go through each f32x2 add/mul/fma; int8 and
//   uint8 values become floats through the 1.5*2^23 magic word built by a byte
//   permute, and codes are packed back from magic words by byte permutes.
// * Adam.  m' = dec(m)*(am*b1) + (1-b1)*g, v' = dec(v)*(av*b2) + (1-b2)*g*g, and
//   a = m' / (bc1*sqrt(v'/bc2) + bc1*eps) with the special-function unit's sqrt
//   and reciprocal.  The residual r' = dec(r)*ar + a*(-lr/ws) + q*(-lr*wd).  These
//   regroup the reference's roundings: every value is within a few ulps of the
//   reference chain, so a code moves by one step only when its value sits within a
//   few ulps of a code boundary (the parity bar allows one LSB on 0.1% of elements).
// * Stochastic rounding (fireflyoptim.py:186-198) in the signed domain:
//   with t = trunc(r'), phi = (r' - t) + sr_bias*tanh(a) and d = phi - copysign(u, r'),
//   dq = t + sign(r') * [d*r' > 0], which is sign(r')*(floor|r'| + [u < clamp(frac|r'|
//   + tanh(a)*sr_bias*sign(r'), 0, 1)]) for |r'| < 2^22 (trunc is the magic add with
//   round-toward-zero).  tanh.approx is good to about 5e-4 relative: where |d| < 2e-4
//   the decision is redone with an accurate tanh.
// * Encode (fireflyoptim.py:22-67): 127/8*log2(1 + 255|x|/absmax) (signed) and
//   255/8*log2(1 + 255 x/absmax) (unsigned) with lg2.approx, rounded by the magic add
//   with the +128 offset folded in (ln(1+y)/ln 256 = log2(1+y)/8).
#pragma once
#include "ff_common.cuh"

namespace ff {
namespace optim {

#ifndef FF_DQT_THREADS
#define FF_DQT_THREADS 384
#endif
constexpr int kThreads = FF_DQT_THREADS;
constexpr int kCtasPerSm = 2;
constexpr int kWarps = kThreads / 32;
constexpr int kBlock = 256;
constexpr int kTabBytes = 256 * 256;  // 256 codes x (32 signed + 32 unsigned copies)
// per warp, two stages of one block's inputs, filled by 1-D bulk (TMA) copies:
// g (512 B) | q (256) | m (256) | v (256) | r (256) | u (1024, supplied-uniform mode only)
// Every warp of a CTA updates one block per iteration (the CTA's kCons consecutive blocks, a
// "chunk"); the chunks' inputs are staged into a ring of CTA stages one chunk ahead, one bulk copy
// per array, by lane 0 of warp i % kCons for the CTA's i-th chunk, so that the staging work is
// spread evenly over the warps (three per scheduler: the warps of a CTA split evenly)
constexpr int kCons = kWarps;
constexpr int kMaxSources = FF_DQT_MAX_SOURCES;
// bytes one block takes in a stage: ng gradient blocks (512 B each; ng = the number of gradient
// sources), q, m, v, r (256 B each), and the uniforms (1 KiB) when they are supplied
__host__ __device__ constexpr int block_stage_bytes(int ng, bool has_u) { return 512 * ng + 1024 + (has_u ? 1024 : 0); }
// stages of the chunk ring (two CTAs of two stages fit an SM)
__host__ __device__ constexpr int num_stages(bool) { return 2; }
// the decode rows, the stages of one chunk each, the stages' full and empty barriers
__host__ __device__ constexpr int smem_bytes_for(int ng, bool has_u, bool multi) {
  return kTabBytes + num_stages(multi) * kCons * block_stage_bytes(ng, has_u) + 2 * num_stages(multi) * 8;
}
__host__ __device__ constexpr int smem_bytes(bool has_u) { return smem_bytes_for(1, has_u, false); }
__host__ __device__ constexpr int smem_bytes_multi(int nsrc) { return smem_bytes_for(nsrc, false, true); }
constexpr float kMagic = 12582912.0f;     // 1.5 * 2^23
// rows with lr / max(ws, eps) above this take the step-by-step chain (see exact_pair)
constexpr float kFastRatio = 16.f;

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
  float den_k, den_c;  // bc1 * sqrt(1/bc2) and bc1 * eps (fp32, correctly rounded sqrt): a's denominator
  uint32_t seed_lo, seed_hi, step_lo, step_hi;
  int64_t rng_offset;
  int64_t row_step, in_row_step;  // grid-stride advance in (rows, elements within a row)
  int bulk;                       // all arrays 16-byte aligned: stage inputs with bulk copies
  // Philox4x32-10 with the counter (call_lo, call_hi, step_lo, step_hi): the round keys, and the
  // first round's products of the constant counter word step_lo
  uint32_t key0[10], key1[10];
  uint32_t r1_hi, r1_lo, r1_c3k;  // mulhi(M1, step_lo), M1 * step_lo, step_hi ^ key1[0]
  const float* u;
  const float* dec_s;
  const float* dec_u;
  // data-parallel mode: the gradient is the average of the nsrc bf16 arrays gsrc[0..nsrc) (summed in
  // fp32 in that order, times inv_nsrc, rounded to bf16); the new weights go to the nqdst arrays
  // qdst[0..nqdst) (q itself among them); gout (or null) receives the averaged gradient
  const uint16_t* gsrc[kMaxSources];
  int8_t* qdst[kMaxSources];
  uint16_t* gout;
  int nsrc, nqdst;
  float inv_nsrc;
};

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void bar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void bar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
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
  const uint64_t t0 = globaltimer_ns(), limit = wait_limit_ns();
  while (!bar_try(bar, parity)) {
    if (globaltimer_ns() - t0 > limit) {
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

__device__ __forceinline__ float sqrt_approx(float x) {
  float y;
  asm("sqrt.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ f2 add2_rz(f2 a, f2 b) {
  f2 r;
  asm("add.rz.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v));
  return r;
}
// max(a, |x|, |y|) for a >= 0 (three-input max)
__device__ __forceinline__ float max3_abs(float a, float x, float y) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(fabsf(x)), "f"(fabsf(y)));
  return r;
}
// maximum over the warp of non-negative floats: their bit patterns order like the values,
// so one integer reduction does it
__device__ __forceinline__ float warp_max_nonneg(float v) {
  return __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(v)));
}
// byte offset c*256 + lane4 of lane l's copy of code c = byte k of w (lane4 = 4*l < 256)
template <int K>
__device__ __forceinline__ uint32_t tab_off(uint32_t w, uint32_t lane4) {
  return __byte_perm(w, lane4, 0x5504u | (K << 4));
}
// the magic word 0x4B4000xx of byte k of w (xx = the byte): its float is 1.5*2^23 + xx
template <int K>
__device__ __forceinline__ float magic_of_byte(uint32_t w) {
  return __uint_as_float(__byte_perm(w, 0x4B400000u, 0x7650u | K));
}
// the low bytes of the magic words of four floats, packed into one word
__device__ __forceinline__ uint32_t pack_magic4(float a, float b, float c, float d) {
  return pack_lo4(__float_as_uint(a), __float_as_uint(b), __float_as_uint(c), __float_as_uint(d));
}
__device__ __forceinline__ uint32_t sign_of(float x) { return __float_as_uint(x) & 0x80000000u; }
__device__ __forceinline__ float with_sign(float mag, uint32_t sign) { return __uint_as_float(__float_as_uint(mag) | sign); }

// x / d with nd = -d and id ~ 1/d: q0 = x*id, r = x - q0*d (exact by FMA), q = q0 + r*id, the
// correctly rounded quotient except extremely close to a rounding midpoint
__device__ __forceinline__ f2 div2(f2 x, f2 nd, f2 id) {
  const f2 q0 = mul2(x, id);
  return fma2(fma2(q0, nd, x), id, q0);
}

// Hyperparameters of the update as fp32 scalars (the roundings of the reference's torch ops).
struct Hyper {
  float neg_lr, beta1, beta2, eps, wd, sr_bias, omb1, omb2, bc1, bc2, ibc1, ibc2;
};

// The reference's chain for one pair of elements, rounding step by step like its torch ops
// (fireflyoptim.py:163-198): used for weight rows whose lr / max(ws, eps) is large, where
// the residual r is large and loses its leading digits when dq is subtracted, so that a
// few ulps of r would move its code.  Inputs: g, the decoded m, v, r (code value times
// block absmax), q (ints), the rows' max(ws, eps) and 1/that, the uniforms.  Outputs the
// new m, v, r and the magic words (1.5*2^23 + q') of the new weights.
__device__ __forceinline__ void exact_pair(const Hyper& h, f2 g, f2 m, f2 v, f2 r, int q0, int q1, float ws0,
                                           float ws1, float iws0, float iws1, float u0, float u1, f2& m_out,
                                           f2& v_out, f2& r_out, f2& q_out) {
  const f2 mone2 = splat(-1.f);
  m = fma2(g, splat(h.omb1), mul2(m, splat(h.beta1)));
  v = fma2(mul2(splat(h.omb2), g), g, mul2(v, splat(h.beta2)));
  const f2 mh = div2(m, splat(-h.bc1), splat(h.ibc1));
  const f2 vh = div2(v, splat(-h.bc2), splat(h.ibc2));
  float vh0, vh1;
  un2(vh, vh0, vh1);
  // sqrt from rsqrt.approx with one residual correction; arguments below 1e-37 (square roots
  // far below eps) use rsqrt(1e-37), so that sqrt(0) = 0 exactly
  const f2 rs = mk2(rsqrt_approx(fmaxf(vh0, 1e-37f)), rsqrt_approx(fmaxf(vh1, 1e-37f)));
  const f2 s0 = mul2(vh, rs);
  const f2 sq = fma2(fma2(s0, mul2(s0, mone2), vh), mul2(rs, splat(0.5f)), s0);
  const f2 den = add2(sq, splat(h.eps));
  float dn0, dn1;
  un2(den, dn0, dn1);
  const f2 a = div2(mh, mul2(den, mone2), mk2(rcp_approx(dn0), rcp_approx(dn1)));
  const f2 qf = mk2((float)q0, (float)q1);
  const f2 ws = mk2(ws0, ws1);
  const f2 dwe = mul2(splat(h.neg_lr), add2(a, mul2(mul2(splat(h.wd), qf), ws)));
  r = add2(r, div2(dwe, mk2(-ws0, -ws1), mk2(iws0, iws1)));
  float r0, r1, a0, a1;
  un2(r, r0, r1);
  un2(a, a0, a1);
  const float rr[2] = {r0, r1}, aa[2] = {a0, a1}, uu[2] = {u0, u1};
  float dqf[2];
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    // floor and frac of |r| (|r| clamped to 2^21, far above any value the update reaches,
    // so that the floor is exact by the magic add with round-down)
    const float absr = fminf(fabsf(rr[e]), 2097152.f);
    const float base = __fsub_rn(__fadd_rd(absr, kMagic), kMagic);
    const float fr = __fsub_rn(absr, base);
    const uint32_t rsign = sign_of(rr[e]);
    float fb = fr;
    if (h.sr_bias != 0.f) {
      const float tb = __fmul_rn(tanh_approx(aa[e]), h.sr_bias);
      fb = __fadd_rn(fr, __uint_as_float(__float_as_uint(tb) ^ rsign));
      if (fabsf(__fsub_rn(uu[e], fb)) < 2e-4f) {
        const float tb2 = __fmul_rn(tanh_accurate(aa[e]), h.sr_bias);
        fb = __fadd_rn(fr, __uint_as_float(__float_as_uint(tb2) ^ rsign));
      }
    }
    const bool up = (uu[e] < fb) && (rr[e] != 0.f);
    dqf[e] = copysignf(up ? __fadd_rn(base, 1.f) : base, rr[e]);
  }
  const int qa = max(-127, min(127, q0 + (__float_as_int(__fadd_rn(dqf[0], kMagic)) - 0x4B400000)));
  const int qb = max(-127, min(127, q1 + (__float_as_int(__fadd_rn(dqf[1], kMagic)) - 0x4B400000)));
  q_out = mk2(__int_as_float(0x4B400000 + qa), __int_as_float(0x4B400000 + qb));
  r_out = sub2(r, mk2(dqf[0], dqf[1]));
  m_out = m;
  v_out = v;
}

// Philox4x32-10 of the counter (c0, c1, step_lo, step_hi) with the launch's round keys; the
// first round's product of the constant counter word comes precomputed
__device__ __forceinline__ void philox_call(uint32_t c0, uint32_t c1, const Params& p, uint32_t (&out)[4]) {
  constexpr uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u;
  uint32_t x0 = p.r1_hi ^ c1 ^ p.key0[0];
  uint32_t x1 = p.r1_lo;
  const uint64_t p0 = (uint64_t)M0 * c0;
  uint32_t x2 = (uint32_t)(p0 >> 32) ^ p.r1_c3k;
  uint32_t x3 = (uint32_t)p0;
#pragma unroll
  for (int r = 1; r < 10; ++r) {
    const uint64_t a = (uint64_t)M0 * x0, b = (uint64_t)M1 * x2;
    x0 = (uint32_t)(b >> 32) ^ x1 ^ p.key0[r];
    x1 = (uint32_t)b;
    x2 = (uint32_t)(a >> 32) ^ x3 ^ p.key1[r];
    x3 = (uint32_t)a;
  }
  out[0] = x0;
  out[1] = x1;
  out[2] = x2;
  out[3] = x3;
}

// decode-table load of the entry at byte offset `off` + IMM of the rows, which start at shared
// address BASE (>= 0: known when compiled, folded into the load's immediate) or `base` (BASE < 0)
template <int BASE, int IMM>
__device__ __forceinline__ float ld_tab(uint32_t base, uint32_t off) {
  float v;
  if constexpr (BASE >= 0)
    asm("ld.shared.f32 %0, [%1+%2];" : "=f"(v) : "r"(off), "n"(BASE + IMM));
  else
    asm("ld.shared.f32 %0, [%1+%2];" : "=f"(v) : "r"(base + off), "n"(IMM));
  return v;
}

// The per-block work of one warp (8 elements per lane).  ROWS: 0 = row_len a multiple of 8 (a
// lane's 8 elements share one weight row), 1 = row_len >= 8 (they span at most two rows),
// 2 = row_len < 8.  TAB: the shared address of the decode rows when known at compile time (the
// kernel dispatches on the usual values), else -1.  MULTI: data-parallel mode (gradient sources
// gsrc, weight destinations qdst; the stage layout of stage_bytes_multi).
template <bool HAS_U, int ROWS, int TAB, bool MULTI>
__device__ __forceinline__ void dqt_run(const Params& p, uint8_t* smem) {
  static_assert(!(HAS_U && MULTI), "supplied uniforms and several gradient sources are not combined");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // a stage holds one chunk (kCons blocks) as regions: the gradient blocks of each source
  // (kCons x 512 B each), then q, m, v, r (kCons x 256 B each), then u (kCons x 1 KiB)
  const int ng = MULTI ? p.nsrc : 1;
  const int chunk_bytes = kCons * block_stage_bytes(ng, HAS_U);
  const int oQ = kCons * 512 * ng, oM = oQ + kCons * 256, oV = oM + kCons * 256, oR = oV + kCons * 256,
            oU = oR + kCons * 256;
  constexpr int NST = num_stages(MULTI);
  uint8_t* stage_p = smem + kTabBytes;
  const uint32_t stage0 = smem_addr(stage_p);
  const uint32_t full0 = stage0 + NST * chunk_bytes, empty0 = full0 + 8 * NST;  // full[NST], empty[NST]
  const uint32_t tab_base = smem_addr(smem);
  const uint32_t lane4 = 4u * lane;
  // data-parallel mode: the averaged gradient of a lane's 8 elements from the sources' words
  // (src(k) returns source k's 4 words), fp32 sums in source order, rounded to bf16
  auto average = [&](auto src, uint32_t (&gw)[4]) {
    f2 acc[4];
    {
      const uint4 w = src(0);
      acc[0] = unpack_bf16x2(w.x); acc[1] = unpack_bf16x2(w.y); acc[2] = unpack_bf16x2(w.z); acc[3] = unpack_bf16x2(w.w);
    }
#pragma unroll
    for (int k = 1; k < kMaxSources; ++k) {
      if (k < p.nsrc) {
        const uint4 w = src(k);
        acc[0] = add2(acc[0], unpack_bf16x2(w.x));
        acc[1] = add2(acc[1], unpack_bf16x2(w.y));
        acc[2] = add2(acc[2], unpack_bf16x2(w.z));
        acc[3] = add2(acc[3], unpack_bf16x2(w.w));
      }
    }
    const f2 inv = splat(p.inv_nsrc);
#pragma unroll
    for (int k = 0; k < 4; ++k) gw[k] = pack_bf16x2(mul2(acc[k], inv));
  };
  const int64_t full_blocks = p.numel / kBlock;  // blocks [0, full_blocks) have 256 elements
  const int64_t nblocks = (p.numel + kBlock - 1) / kBlock;
  const int64_t staged_blocks = p.bulk ? full_blocks : 0;
  const int64_t wstride = (int64_t)gridDim.x * kCons;  // blocks between a warp's iterations
  const float eps = p.eps;
  const int64_t last_row = (p.elem_base + p.numel - 1) / p.row_len;
  const Hyper hy{p.neg_lr, p.beta1, p.beta2, eps, p.wd, p.sr_bias, p.omb1, p.omb2, p.bc1, p.bc2, p.ibc1, p.ibc2};

  // One block: inputs as packed words (g bf16 pairs; q, m, v, r bytes), uniforms, the weight rows'
  // max(ws, eps) and where the second row starts (jsw), the block absmax; writes nvalid elements.
  auto process = [&](int64_t blk, const uint32_t (&gw)[4], const uint32_t (&qw)[2], const uint32_t (&mw)[2],
                     const uint32_t (&vw)[2], const uint32_t (&rw)[2], const float* u, float wsa, float wsb,
                     int jsw, float am, float av, float ar, int nvalid) {
    const int64_t e0 = blk * kBlock + lane * 8;
    uint32_t rw4[4];  // Philox output: 16 bits per element
    if constexpr (!HAS_U) {
      const uint64_t call = (uint64_t)(p.rng_offset + e0) >> 3;
      philox_call((uint32_t)call, (uint32_t)(call >> 32), p, rw4);
    }
    const float caa = __fmul_rn(p.neg_lr, rcp_approx(wsa)), cab = __fmul_rn(p.neg_lr, rcp_approx(wsb));
    // rows with a large lr/ws carry large residuals: they take the step-by-step chain
    const bool exact = ROWS == 2 || fabsf(caa) > kFastRatio || fabsf(cab) > kFastRatio;
    const uint32_t qb[2] = {qw[0] ^ 0x80808080u, qw[1] ^ 0x80808080u};  // bytes biased by 128
    // decode of pair pp (fireflyoptim.py:39-80): one permute + one shared load per code
    auto decode = [&](int pp, f2& tm, f2& tv, f2& tr, f2& qm) {
      const int w = pp >> 1;
      uint32_t om0, om1, ov0, ov1, or0, or1;
      float qm0, qm1;
      if (pp & 1) {
        om0 = tab_off<2>(mw[w], lane4); om1 = tab_off<3>(mw[w], lane4);
        ov0 = tab_off<2>(vw[w], lane4); ov1 = tab_off<3>(vw[w], lane4);
        or0 = tab_off<2>(rw[w], lane4); or1 = tab_off<3>(rw[w], lane4);
        qm0 = magic_of_byte<2>(qb[w]); qm1 = magic_of_byte<3>(qb[w]);
      } else {
        om0 = tab_off<0>(mw[w], lane4); om1 = tab_off<1>(mw[w], lane4);
        ov0 = tab_off<0>(vw[w], lane4); ov1 = tab_off<1>(vw[w], lane4);
        or0 = tab_off<0>(rw[w], lane4); or1 = tab_off<1>(rw[w], lane4);
        qm0 = magic_of_byte<0>(qb[w]); qm1 = magic_of_byte<1>(qb[w]);
      }
      tm = mk2(ld_tab<TAB, 0>(tab_base, om0), ld_tab<TAB, 0>(tab_base, om1));
      tv = mk2(ld_tab<TAB, 128>(tab_base, ov0), ld_tab<TAB, 128>(tab_base, ov1));
      tr = mk2(ld_tab<TAB, 0>(tab_base, or0), ld_tab<TAB, 0>(tab_base, or1));
      qm = mk2(qm0, qm1);
    };
    auto uniforms = [&](int pp, float& u0, float& u1) {
      if constexpr (HAS_U) {
        u0 = u[2 * pp];
        u1 = u[2 * pp + 1];
      } else {
        // u = (h + 0.5) / 65536 for the 16-bit halves h of the Philox word: 2^23 + h is built by a
        // byte permute, and (2^23 + h) * 2^-16 + (2^-17 - 128) is exact in one FMA
        const uint32_t wd_ = rw4[pp];
        u0 = __fmaf_rn(__int_as_float(__byte_perm(wd_, 0x4B000000u, 0x7610)), 1.0f / 65536.0f, 1.0f / 131072.0f - 128.0f);
        u1 = __fmaf_rn(__int_as_float(__byte_perm(wd_, 0x4B000000u, 0x7632)), 1.0f / 65536.0f, 1.0f / 131072.0f - 128.0f);
      }
    };
    f2 mn[4], vn[4], rn[4], qn[4];
    if (!exact) {
      const f2 am2 = splat(am * p.beta1), av2 = splat(av * p.beta2), ar2 = splat(ar);
      const f2 den_k = splat(p.den_k), den_c = splat(p.den_c);  // bc1*sqrt(v/bc2) + bc1*eps
#pragma unroll
      for (int pp = 0; pp < 4; ++pp) {
        const int j0 = 2 * pp, j1 = 2 * pp + 1;
        const float ca0 = j0 < jsw ? caa : cab, ca1 = j1 < jsw ? caa : cab;
        f2 tm, tv, tr, qm;
        decode(pp, tm, tv, tr, qm);
        const f2 g = mk2(__uint_as_float(gw[pp] << 16), __uint_as_float(gw[pp] & 0xFFFF0000u));
        // Adam moments (fireflyoptim.py:175-182)
        const f2 m = fma2(tm, am2, mul2(g, splat(p.omb1)));
        const f2 v = fma2(tv, av2, mul2(mul2(g, g), splat(p.omb2)));
        float v0, v1;
        un2(v, v0, v1);
        float d0, d1;
        un2(fma2(mk2(sqrt_approx(v0), sqrt_approx(v1)), den_k, den_c), d0, d1);
        const f2 a = mul2(m, mk2(rcp_approx(d0), rcp_approx(d1)));
        // DQT residual (fireflyoptim.py:180-184)
        const f2 qf = sub2(qm, splat(kMagic + 128.f));
        const f2 r = fma2(tr, ar2, fma2(a, mk2(ca0, ca1), mul2(qf, splat(p.neg_lr * p.wd))));
        // momentum-biased stochastic rounding (fireflyoptim.py:186-198)
        float r0, r1, a0, a1;
        un2(r, r0, r1);
        un2(a, a0, a1);
        const uint32_t s0 = sign_of(r0), s1 = sign_of(r1);
        const f2 ms = mk2(with_sign(kMagic, s0), with_sign(kMagic, s1));
        const f2 rt = sub2(add2_rz(r, ms), ms);  // trunc(r) for |r| < 2^22
        float uj0, uj1;
        uniforms(pp, uj0, uj1);
        // sr_bias * tanh(a) = sr_bias - 2 sr_bias / (1 + e^{2a}) (absolute error about 1e-7)
        float e0_, e1_;
        un2(mul2(a, splat(2.8853900817779268f)), e0_, e1_);  // 2a / ln 2
        float w0, w1;
        un2(add2(mk2(ex2_approx(e0_), ex2_approx(e1_)), splat(1.f)), w0, w1);
        const f2 phi = fma2(mk2(rcp_approx(w0), rcp_approx(w1)), splat(-2.f * p.sr_bias),
                            add2(sub2(r, rt), splat(p.sr_bias)));
        const f2 us = mk2(with_sign(uj0, s0), with_sign(uj1, s1));
        float p0, p1;
        un2(mul2(sub2(phi, us), r), p0, p1);
        // dq = trunc(r) + sign(r) * [u < threshold]  (d*r > 0: u on the rounding-up side, r != 0)
        const f2 inc = mk2(p0 > 0.f ? with_sign(1.f, s0) : 0.f, p1 > 0.f ? with_sign(1.f, s1) : 0.f);
        const f2 dq = add2(rt, inc);
        float qs0, qs1;
        un2(add2(qf, dq), qs0, qs1);
        qn[pp] = add2(mk2(fminf(fmaxf(qs0, -127.f), 127.f), fminf(fmaxf(qs1, -127.f), 127.f)), splat(kMagic));
        rn[pp] = sub2(r, dq);
        mn[pp] = m;
        vn[pp] = v;
      }
    } else {
      const f2 am2 = splat(am), av2 = splat(av), ar2 = splat(ar);
#pragma unroll
      for (int pp = 0; pp < 4; ++pp) {
        const int j0 = 2 * pp, j1 = 2 * pp + 1;
        float ws0 = j0 < jsw ? wsa : wsb, ws1 = j1 < jsw ? wsa : wsb;
        if constexpr (ROWS == 2) {  // rows shorter than 8 elements: one lookup per element
          ws0 = fmaxf(__ldg(p.wscale + min64((p.elem_base + min64(e0 + j0, p.numel - 1)) / p.row_len, last_row)), eps);
          ws1 = fmaxf(__ldg(p.wscale + min64((p.elem_base + min64(e0 + j1, p.numel - 1)) / p.row_len, last_row)), eps);
        }
        f2 tm, tv, tr, qm;
        decode(pp, tm, tv, tr, qm);
        float qm0, qm1;
        un2(qm, qm0, qm1);
        const int q0 = (int)(__float_as_uint(qm0) & 0xFFu) - 128, q1 = (int)(__float_as_uint(qm1) & 0xFFu) - 128;
        const f2 g = mk2(__uint_as_float(gw[pp] << 16), __uint_as_float(gw[pp] & 0xFFFF0000u));
        float uj0, uj1;
        uniforms(pp, uj0, uj1);
        exact_pair(hy, g, mul2(tm, am2), mul2(tv, av2), mul2(tr, ar2), q0, q1, ws0, ws1, __frcp_rn(ws0),
                   __frcp_rn(ws1), uj0, uj1, mn[pp], vn[pp], rn[pp], qn[pp]);
      }
    }
    // ---------------- block absmax and re-encode (mu-law, fireflyoptim.py:22-67)
    float xm = 0.f, xv = 0.f, xr = 0.f;
#pragma unroll
    for (int pp = 0; pp < 4; ++pp) {
      float a0, a1;
      un2(mn[pp], a0, a1);
      xm = max3_abs(xm, a0, a1);
      un2(vn[pp], a0, a1);
      xv = max3_abs(xv, a0, a1);  // v >= 0; |.| turns -0 into +0
      un2(rn[pp], a0, a1);
      xr = max3_abs(xr, a0, a1);
    }
    xm = fmaxf(warp_max_nonneg(xm), 1e-12f);
    xv = fmaxf(warp_max_nonneg(xv), 1e-12f);
    xr = fmaxf(warp_max_nonneg(xr), 1e-12f);
    // 255 / absmax: |x| * this is 255 * |x| / absmax (within an ulp or two)
    const float km = __fmul_rn(255.f, rcp_approx(xm)), kr = __fmul_rn(255.f, rcp_approx(xr));
    const f2 kv = splat(__fmul_rn(255.f, rcp_approx(xv)));
    float cm[8], cv[8], cr[8], cq[8];
    // |x| / absmax can exceed 1 by an ulp (absmax is the largest |x|); log2(256 + tiny) * 127/8
    // still rounds to 127 (255 for v), so no clamps are needed.  v is never negative.
#pragma unroll
    for (int pp = 0; pp < 4; ++pp) {
      float x0, x1, y0, y1, z0, z1;
      un2(mn[pp], x0, x1);
      un2(rn[pp], y0, y1);
      // signed m and r: code = 128 + sign(x) * rint(127/8 * log2(1 + 255 |x| / absmax))
      float lm0, lm1, lr0, lr1;
      un2(add2(mk2(__fmul_rn(fabsf(x0), km), __fmul_rn(fabsf(x1), km)), splat(1.f)), lm0, lm1);
      un2(add2(mk2(__fmul_rn(fabsf(y0), kr), __fmul_rn(fabsf(y1), kr)), splat(1.f)), lr0, lr1);
      un2(fma2(mk2(with_sign(lg2_approx(lm0), sign_of(x0)), with_sign(lg2_approx(lm1), sign_of(x1))),
               splat(15.875f), splat(kMagic + 128.f)),
          cm[2 * pp], cm[2 * pp + 1]);
      un2(fma2(mk2(with_sign(lg2_approx(lr0), sign_of(y0)), with_sign(lg2_approx(lr1), sign_of(y1))),
               splat(15.875f), splat(kMagic + 128.f)),
          cr[2 * pp], cr[2 * pp + 1]);
      // unsigned v: code = rint(255/8 * log2(1 + 255 v / absmax))
      un2(fma2(vn[pp], kv, splat(1.f)), z0, z1);
      un2(fma2(mk2(lg2_approx(z0), lg2_approx(z1)), splat(31.875f), splat(kMagic)), cv[2 * pp], cv[2 * pp + 1]);
      un2(qn[pp], cq[2 * pp], cq[2 * pp + 1]);
    }
    if (nvalid == 8) {
      // generic-proxy stores; the bulk copies only ever read other blocks
      const uint2 qv = make_uint2(pack_magic4(cq[0], cq[1], cq[2], cq[3]), pack_magic4(cq[4], cq[5], cq[6], cq[7]));
      if constexpr (MULTI) {  // every rank's copy of the weights (peers' over NVLink)
#pragma unroll
        for (int k = 0; k < kMaxSources; ++k)
          if (k < p.nqdst) *reinterpret_cast<uint2*>(p.qdst[k] + e0) = qv;
      } else {
        *reinterpret_cast<uint2*>(p.q + e0) = qv;
      }
      *reinterpret_cast<uint2*>(p.m_q + e0) = make_uint2(pack_magic4(cm[0], cm[1], cm[2], cm[3]), pack_magic4(cm[4], cm[5], cm[6], cm[7]));
      *reinterpret_cast<uint2*>(p.v_q + e0) = make_uint2(pack_magic4(cv[0], cv[1], cv[2], cv[3]), pack_magic4(cv[4], cv[5], cv[6], cv[7]));
      *reinterpret_cast<uint2*>(p.r_q + e0) = make_uint2(pack_magic4(cr[0], cr[1], cr[2], cr[3]), pack_magic4(cr[4], cr[5], cr[6], cr[7]));
    } else {
      for (int j = 0; j < nvalid; ++j) {
        if constexpr (MULTI) {
          for (int k = 0; k < p.nqdst; ++k) p.qdst[k][e0 + j] = (int8_t)__float_as_uint(cq[j]);
        } else {
          p.q[e0 + j] = (int8_t)__float_as_uint(cq[j]);
        }
        p.m_q[e0 + j] = (uint8_t)__float_as_uint(cm[j]);
        p.v_q[e0 + j] = (uint8_t)__float_as_uint(cv[j]);
        p.r_q[e0 + j] = (uint8_t)__float_as_uint(cr[j]);
      }
    }
    if (lane == 0) {
      p.m_absmax[blk] = xm;
      p.v_absmax[blk] = xv;
      p.r_absmax[blk] = xr;
    }
  };

  // ---- staged loop: chunks of kCons consecutive full blocks; iteration it of this CTA is chunk
  // blockIdx.x + it * gridDim.x, staged into stage it % NST
  const int64_t staged_chunks = p.bulk ? (full_blocks + kCons - 1) / kCons : 0;
  // lane 0 of warp it % kCons: stage the chunk of iteration it (if any) into stage it % NST once
  // every warp has read that stage's previous chunk (iteration it - NST); false if that wait gave up
  auto produce = [&](int it) -> bool {
    const int64_t c = (int64_t)blockIdx.x + (int64_t)it * gridDim.x;
    if (c >= staged_chunks) return true;
    const int st = it % NST;
    if (it >= NST && !bar_wait(empty0 + 8 * st, ((it / NST) & 1) ^ 1)) return false;
    const int64_t b0 = c * kCons;
    const int nb = (int)min64(kCons, full_blocks - b0);
    const uint32_t dst = stage0 + st * chunk_bytes, bar = full0 + 8 * st;
    const int64_t e = b0 * kBlock;
    bar_expect(bar, (uint32_t)(nb * block_stage_bytes(ng, HAS_U)));
    if constexpr (MULTI) {  // every source's gradient blocks (peers' over NVLink, no multicast)
#pragma unroll
      for (int k = 0; k < kMaxSources; ++k)
        if (k < p.nsrc) bulk_g2s(dst + k * kCons * 512, p.gsrc[k] + e, nb * 512, bar);
    } else {
      bulk_g2s(dst, p.g + e, nb * 512, bar);
    }
    bulk_g2s(dst + oQ, p.q + e, nb * 256, bar);
    bulk_g2s(dst + oM, p.m_q + e, nb * 256, bar);
    bulk_g2s(dst + oV, p.v_q + e, nb * 256, bar);
    bulk_g2s(dst + oR, p.r_q + e, nb * 256, bar);
    if constexpr (HAS_U) bulk_g2s(dst + oU, p.u + e, nb * 1024, bar);
    return true;
  };
  for (int k = 0; k < NST - 1; ++k)
    if (lane == 0 && warp == k % kCons) produce(k);
  int64_t blk = (int64_t)blockIdx.x * kCons + warp;
  // weight row of this lane's first element, advanced incrementally (no division per block)
  int64_t row, in_row;
  {
    const int64_t ge = p.elem_base + blk * kBlock + lane * 8;
    row = ge / p.row_len;
    in_row = ge - row * p.row_len;
  }
  float am = 0.f, av = 0.f, ar = 0.f;
  if (blk < full_blocks && staged_chunks > 0) {
    am = __ldg(p.m_absmax + blk);
    av = __ldg(p.v_absmax + blk);
    ar = __ldg(p.r_absmax + blk);
  }
  for (int it = 0;; ++it) {
    const int64_t c = (int64_t)blockIdx.x + (int64_t)it * gridDim.x;
    if (c >= staged_chunks) break;
    if (lane == 0 && warp == (it + NST - 1) % kCons && !produce(it + NST - 1)) return;  // NST - 1 chunks ahead
    const int st = it % NST;
    blk = c * kCons + warp;
    const bool mine = blk < full_blocks;  // only the last chunk can hold fewer than kCons blocks
    const int64_t nxt = blk + wstride;
    const float am_c = am, av_c = av, ar_c = ar;
    if (nxt < full_blocks) {  // the next block's absmax, one iteration ahead
      am = __ldg(p.m_absmax + nxt);
      av = __ldg(p.v_absmax + nxt);
      ar = __ldg(p.r_absmax + nxt);
    }
    const int64_t ra = min64(row, last_row), rb = min64(row + 1, last_row);
    const int jsw = ROWS != 1 ? 8 : (int)min64(8, p.row_len - in_row);  // j >= jsw: next row
    const float wsa = fmaxf(__ldg(p.wscale + ra), eps);
    const float wsb = jsw < 8 ? fmaxf(__ldg(p.wscale + rb), eps) : wsa;
    uint32_t gw[4], qw[2], mw[2], vw[2], rw[2];
    float u[HAS_U ? 8 : 1];
    if (mine) {
      if (!bar_wait(full0 + 8 * st, (it / NST) & 1)) return;  // copies lost: status raised
      const uint8_t* sb = stage_p + st * chunk_bytes;
      if constexpr (MULTI) {
        average([&](int k) { return *reinterpret_cast<const uint4*>(sb + k * kCons * 512 + warp * 512 + lane * 16); },
                gw);
        if (p.gout) *reinterpret_cast<uint4*>(p.gout + blk * kBlock + lane * 8) = make_uint4(gw[0], gw[1], gw[2], gw[3]);
      } else {
        const uint4 g4 = *reinterpret_cast<const uint4*>(sb + warp * 512 + lane * 16);
        gw[0] = g4.x; gw[1] = g4.y; gw[2] = g4.z; gw[3] = g4.w;
      }
      const uint2 q2 = *reinterpret_cast<const uint2*>(sb + oQ + warp * 256 + lane * 8);
      const uint2 m2 = *reinterpret_cast<const uint2*>(sb + oM + warp * 256 + lane * 8);
      const uint2 v2 = *reinterpret_cast<const uint2*>(sb + oV + warp * 256 + lane * 8);
      const uint2 r2 = *reinterpret_cast<const uint2*>(sb + oR + warp * 256 + lane * 8);
      qw[0] = q2.x; qw[1] = q2.y; mw[0] = m2.x; mw[1] = m2.y;
      vw[0] = v2.x; vw[1] = v2.y; rw[0] = r2.x; rw[1] = r2.y;
      if constexpr (HAS_U) {
        const float4 u0 = *reinterpret_cast<const float4*>(sb + oU + warp * 1024 + lane * 32);
        const float4 u1 = *reinterpret_cast<const float4*>(sb + oU + warp * 1024 + lane * 32 + 16);
        u[0] = u0.x; u[1] = u0.y; u[2] = u0.z; u[3] = u0.w;
        u[4] = u1.x; u[5] = u1.y; u[6] = u1.z; u[7] = u1.w;
      }
    }
    __syncwarp();  // every lane has its inputs: this warp's part of the stage may be refilled
    if (lane == 0) bar_arrive(empty0 + 8 * st);
    if (!mine) break;  // the last chunk, and this warp has no block in it
    process(blk, gw, qw, mw, vw, rw, u, wsa, wsb, jsw, am_c, av_c, ar_c, 8);
    row += p.row_step;
    in_row += p.in_row_step;
    if (in_row >= p.row_len) {
      in_row -= p.row_len;
      ++row;
    }
  }
  blk = (p.bulk ? full_blocks : 0) + (int64_t)blockIdx.x * kCons + warp;
  // ---- the rest: the ragged last block, or every block when the arrays are not 16-byte aligned
  for (; blk < nblocks; blk += wstride) {
    const int64_t e0 = blk * kBlock + lane * 8;
    const int nvalid = (int)max64(0, min64(8, p.numel - e0));
    uint32_t gw[4], qw[2], mw[2], vw[2], rw[2];
    float u[HAS_U ? 8 : 1];
    if (nvalid == 8) {
      if constexpr (MULTI) {  // plain loads: the peers' arrays are not read-only data of this kernel
        average([&](int k) { return *reinterpret_cast<const uint4*>(p.gsrc[k] + e0); }, gw);
      } else {
        const uint4 g4 = __ldg(reinterpret_cast<const uint4*>(p.g + e0));
        gw[0] = g4.x; gw[1] = g4.y; gw[2] = g4.z; gw[3] = g4.w;
      }
      const uint2 q2 = *reinterpret_cast<const uint2*>(p.q + e0);
      const uint2 m2 = *reinterpret_cast<const uint2*>(p.m_q + e0);
      const uint2 v2 = *reinterpret_cast<const uint2*>(p.v_q + e0);
      const uint2 r2 = *reinterpret_cast<const uint2*>(p.r_q + e0);
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
          if constexpr (!MULTI) gw[j >> 1] |= (uint32_t)p.g[e0 + j] << (16 * (j & 1));
          qw[w] |= ((uint32_t)(uint8_t)p.q[e0 + j]) << sh;
          mw[w] = (mw[w] & ~(0xFFu << sh)) | ((uint32_t)p.m_q[e0 + j] << sh);
          vw[w] |= (uint32_t)p.v_q[e0 + j] << sh;
          rw[w] = (rw[w] & ~(0xFFu << sh)) | ((uint32_t)p.r_q[e0 + j] << sh);
        }
        if constexpr (HAS_U) u[j] = j < nvalid ? __ldg(p.u + e0 + j) : 2.f;
      }
      if constexpr (MULTI) {  // the same average, missing elements 0 in every source
        average([&](int k) {
          uint32_t w[4] = {0u, 0u, 0u, 0u};
          for (int j = 0; j < nvalid; ++j) w[j >> 1] |= (uint32_t)p.gsrc[k][e0 + j] << (16 * (j & 1));
          return make_uint4(w[0], w[1], w[2], w[3]);
        }, gw);
      }
    }
    if constexpr (MULTI) {
      if (p.gout) {
        for (int j = 0; j < nvalid; ++j) p.gout[e0 + j] = (uint16_t)(gw[j >> 1] >> (16 * (j & 1)));
      }
    }
    const int64_t ge = p.elem_base + min64(e0, p.numel - 1);
    const int64_t r0 = ge / p.row_len, in0 = ge - r0 * p.row_len;
    const int64_t ra = min64(r0, last_row), rb = min64(r0 + 1, last_row);
    const int jsw = ROWS != 1 ? 8 : (int)min64(8, p.row_len - in0);
    const float wsa = fmaxf(__ldg(p.wscale + ra), eps);
    const float wsb = jsw < 8 ? fmaxf(__ldg(p.wscale + rb), eps) : wsa;
    process(blk, gw, qw, mw, vw, rw, u, wsa, wsb, jsw, __ldg(p.m_absmax + blk), __ldg(p.v_absmax + blk),
            __ldg(p.r_absmax + blk), nvalid);
  }
}

template <bool HAS_U, int ROWS, bool MULTI>
__global__ void __launch_bounds__(kThreads, HAS_U ? 1 : kCtasPerSm) dqt_adamw8_kernel(Params p) {
  extern __shared__ __align__(1024) uint8_t smem[];  // decode rows, then the two stages, then barriers
  // decode rows: word 64*c + l = signed entry of code c, word 64*c + 32 + l = unsigned entry
  {
    float* tw = reinterpret_cast<float*>(smem);
    for (int i = threadIdx.x; i < kTabBytes / 4; i += kThreads) {
      const int c = i >> 6;
      tw[i] = (i & 32) ? __ldg(p.dec_u + c) : __ldg(p.dec_s + c);
    }
  }
  if (threadIdx.x == 0) {  // full[]: the producer's arrival with the bytes; empty[]: one arrival per consumer warp
    constexpr int NST = num_stages(MULTI);
    const int chunk_bytes = kCons * block_stage_bytes(MULTI ? p.nsrc : 1, HAS_U);
    const uint32_t full0 = smem_addr(smem + kTabBytes + NST * chunk_bytes);
    for (int k = 0; k < NST; ++k) {
      bar_init(full0 + 8 * k, 1);
      bar_init(full0 + 8 * (NST + k), kCons);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  const uint32_t base = smem_addr(smem);
  if (base == 0)
    dqt_run<HAS_U, ROWS, 0, MULTI>(p, smem);
  else if (base == 1024)
    dqt_run<HAS_U, ROWS, 1024, MULTI>(p, smem);
  else
    dqt_run<HAS_U, ROWS, -1, MULTI>(p, smem);
  // the weights stored into the peers' memory are visible to them once the kernel has ended (the
  // host orders the peers' next reads after it with a collective)
  if constexpr (MULTI) __threadfence_system();
}

}  // namespace optim
}  // namespace ff


namespace ff {
namespace optim {

// One launch of the update over `numel` elements.  nsrc == 0: the single-source kernel (g; u for
// supplied uniforms); nsrc >= 1: the data-parallel kernel (gradient sources gsrc, weight
// destinations qdst, optional averaged-gradient output gout).
inline int dqt_launch(const char* name, int8_t* q, const float* wscale, int64_t row_len, int64_t elem_base,
                      const uint16_t* g, uint8_t* m_q, float* m_absmax, uint8_t* v_q, float* v_absmax, uint8_t* r_q,
                      float* r_absmax, int64_t numel, int64_t block, double lr, double beta1, double beta2,
                      double eps, double wd, double bc1, double bc2, double sr_bias, uint64_t seed, uint64_t step,
                      int64_t rng_offset, const float* u, const float* dec_s, const float* dec_u,
                      const uint16_t* const* gsrc, int nsrc, int8_t* const* qdst, int nqdst, uint16_t* gout,
                      void* stream) {
  const bool multi = nsrc > 0;
  FF_REQUIRE(numel >= 0 && row_len >= 1 && elem_base >= 0 && rng_offset >= 0, FF_ERR_INVALID_ARG, "%s: bad sizes",
             name);
  FF_REQUIRE(block == kBlock, FF_ERR_UNSUPPORTED, "%s: block must be %d (got %lld)", name, kBlock, (long long)block);
  FF_REQUIRE(nsrc >= 0 && nsrc <= kMaxSources && (!multi || (nqdst >= 1 && nqdst <= kMaxSources)),
             FF_ERR_INVALID_ARG, "%s: %d gradient sources and %d weight destinations (1 to %d each)", name, nsrc,
             nqdst, kMaxSources);
  if (numel == 0) return FF_OK;
  FF_REQUIRE(q && wscale && (multi || g) && m_q && m_absmax && v_q && v_absmax && r_q && r_absmax && dec_s && dec_u,
             FF_ERR_INVALID_ARG, "%s: null pointer", name);
  FF_REQUIRE((multi || aligned(g, 16)) && aligned(q, 8) && aligned(m_q, 8) && aligned(v_q, 8) && aligned(r_q, 8),
             FF_ERR_UNSUPPORTED, "%s: g needs 16-byte and code arrays 8-byte alignment", name);
  for (int k = 0; k < nsrc; ++k) {
    FF_REQUIRE(gsrc[k], FF_ERR_INVALID_ARG, "%s: null gradient source %d", name, k);
    FF_REQUIRE(aligned(gsrc[k], 16), FF_ERR_UNSUPPORTED, "%s: gradient source %d needs 16-byte alignment", name, k);
  }
  for (int k = 0; multi && k < nqdst; ++k) {
    FF_REQUIRE(qdst[k], FF_ERR_INVALID_ARG, "%s: null weight destination %d", name, k);
    FF_REQUIRE(aligned(qdst[k], 8), FF_ERR_UNSUPPORTED, "%s: weight destination %d needs 8-byte alignment", name, k);
  }
  FF_REQUIRE(!gout || aligned(gout, 16), FF_ERR_UNSUPPORTED, "%s: the averaged-gradient output needs 16-byte alignment",
             name);
  FF_REQUIRE(!(multi && u), FF_ERR_UNSUPPORTED, "%s: supplied uniforms take a single gradient source", name);
  FF_REQUIRE(rng_offset % 8 == 0, FF_ERR_UNSUPPORTED, "%s: rng_offset must be a multiple of 8", name);
  FF_REQUIRE(bc1 > 0.0 && bc2 > 0.0, FF_ERR_INVALID_ARG, "%s: bias corrections must be > 0", name);
  Params p;
  p.q = q;
  p.wscale = wscale;
  p.row_len = row_len;
  p.elem_base = elem_base;
  p.g = multi ? gsrc[0] : g;
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
  // the same fp32 roundings as the device expression p.bc1 * sqrtf(p.ibc2), p.bc1 * p.eps
  {
    volatile float sq = sqrtf(p.ibc2);  // IEEE sqrt, correctly rounded as on the device
    p.den_k = (float)(p.bc1 * sq);
    p.den_c = (float)(p.bc1 * p.eps);
  }
  p.seed_lo = (uint32_t)seed;
  p.seed_hi = (uint32_t)(seed >> 32);
  p.step_lo = (uint32_t)step;
  p.step_hi = (uint32_t)(step >> 32);
  for (int r = 0; r < 10; ++r) {  // Philox4x32-10 key schedule (Weyl increments)
    p.key0[r] = p.seed_lo + (uint32_t)r * 0x9E3779B9u;
    p.key1[r] = p.seed_hi + (uint32_t)r * 0xBB67AE85u;
  }
  {
    const uint64_t prod = (uint64_t)0xCD9E8D57u * (uint64_t)p.step_lo;
    p.r1_hi = (uint32_t)(prod >> 32);
    p.r1_lo = (uint32_t)prod;
    p.r1_c3k = p.step_hi ^ p.key1[0];
  }
  p.rng_offset = rng_offset;
  p.u = u;
  p.dec_s = dec_s;
  p.dec_u = dec_u;
  for (int k = 0; k < kMaxSources; ++k) {
    p.gsrc[k] = k < nsrc ? gsrc[k] : nullptr;
    p.qdst[k] = multi && k < nqdst ? qdst[k] : nullptr;
  }
  p.gout = gout;
  p.nsrc = nsrc;
  p.nqdst = multi ? nqdst : 0;
  p.inv_nsrc = multi ? (float)(1.0 / nsrc) : 1.f;
  // bulk staging needs every staged array 16-byte aligned (the sources were checked above)
  p.bulk = aligned(q, 16) && aligned(m_q, 16) && aligned(v_q, 16) && aligned(r_q, 16) && (!u || aligned(u, 16));
  int dev = 0;
  cudaGetDevice(&dev);
  static bool attr_set[64] = {false};
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    const void* fns_u[] = {(const void*)dqt_adamw8_kernel<true, 0, false>, (const void*)dqt_adamw8_kernel<true, 1, false>,
                           (const void*)dqt_adamw8_kernel<true, 2, false>};
    const void* fns[] = {(const void*)dqt_adamw8_kernel<false, 0, false>, (const void*)dqt_adamw8_kernel<false, 1, false>,
                         (const void*)dqt_adamw8_kernel<false, 2, false>};
    const void* fns_m[] = {(const void*)dqt_adamw8_kernel<false, 0, true>, (const void*)dqt_adamw8_kernel<false, 1, true>,
                           (const void*)dqt_adamw8_kernel<false, 2, true>};
    for (const void* fn : fns_u)
      FF_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes(true)),
                  "ff_dqt_adamw8 smem attribute");
    for (const void* fn : fns)
      FF_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes(false)),
                  "ff_dqt_adamw8 smem attribute");
    for (const void* fn : fns_m)
      FF_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes_multi(kMaxSources)),
                  "ff_dqt_adamw8 smem attribute");
    attr_set[dev] = true;
  }
  const int64_t nblocks = (numel + kBlock - 1) / kBlock;
  int nsm = 148;
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  int smem_sm = 0;
  cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
  const int smem = u ? smem_bytes(true) : multi ? smem_bytes_multi(nsrc) : smem_bytes(false);
  // CTAs per SM: two unless their shared memory (plus the 1 KiB the runtime reserves per CTA) does not fit
  const int per_sm = u ? 1 : (2 * (smem + 1024) <= smem_sm ? kCtasPerSm : 1);
  const int64_t want = (nblocks + kCons - 1) / kCons;
  const int grid = (int)min64(want, (int64_t)nsm * per_sm);
  const int64_t stride_elems = (int64_t)grid * kCons * kBlock;
  p.row_step = stride_elems / row_len;
  p.in_row_step = stride_elems % row_len;
  cudaStream_t st = as_stream(stream);
  // a lane's 8 elements start at a multiple of 8 of the weight when elem_base is one
  const int rows_mode = (row_len % 8 == 0 && elem_base % 8 == 0) ? 0 : (row_len >= 8 ? 1 : 2);
#define FF_DQT_LAUNCH(HU, RM, MU) dqt_adamw8_kernel<HU, RM, MU><<<grid, kThreads, smem, st>>>(p)
  if (u) {
    if (rows_mode == 0) FF_DQT_LAUNCH(true, 0, false);
    else if (rows_mode == 1) FF_DQT_LAUNCH(true, 1, false);
    else FF_DQT_LAUNCH(true, 2, false);
  } else if (multi) {
    if (rows_mode == 0) FF_DQT_LAUNCH(false, 0, true);
    else if (rows_mode == 1) FF_DQT_LAUNCH(false, 1, true);
    else FF_DQT_LAUNCH(false, 2, true);
  } else {
    if (rows_mode == 0) FF_DQT_LAUNCH(false, 0, false);
    else if (rows_mode == 1) FF_DQT_LAUNCH(false, 1, false);
    else FF_DQT_LAUNCH(false, 2, false);
  }
#undef FF_DQT_LAUNCH
  return check_launch(name);
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
  return ff::optim::dqt_launch("ff_dqt_adamw8", q, wscale, row_len, elem_base, g, m_q, m_absmax, v_q, v_absmax, r_q,
                               r_absmax, numel, block, lr, beta1, beta2, eps, wd, bc1, bc2, sr_bias, seed, step,
                               rng_offset, u, dec_s, dec_u, nullptr, 0, nullptr, 0, nullptr, stream);
}

extern "C" int ff_dqt_adamw8_peers(int8_t* q, const float* wscale, int64_t row_len, int64_t elem_base,
                                   const uint16_t* const* g_srcs, int n_srcs, int8_t* const* q_dsts, int n_dsts,
                                   uint16_t* g_out, uint8_t* m_q, float* m_absmax, uint8_t* v_q, float* v_absmax,
                                   uint8_t* r_q, float* r_absmax, int64_t numel, int64_t block, double lr,
                                   double beta1, double beta2, double eps, double wd, double bc1, double bc2,
                                   double sr_bias, uint64_t seed, uint64_t step, int64_t rng_offset,
                                   const float* dec_s, const float* dec_u, void* stream) {
  using namespace ff;
  FF_REQUIRE(g_srcs && q_dsts && n_srcs >= 1, FF_ERR_INVALID_ARG, "ff_dqt_adamw8_peers: no gradient sources");
  return ff::optim::dqt_launch("ff_dqt_adamw8_peers", q, wscale, row_len, elem_base, nullptr, m_q, m_absmax, v_q,
                               v_absmax, r_q, r_absmax, numel, block, lr, beta1, beta2, eps, wd, bc1, bc2, sr_bias,
                               seed, step, rng_offset, nullptr, dec_s, dec_u, g_srcs, n_srcs, q_dsts, n_dsts, g_out,
                               stream);
}
