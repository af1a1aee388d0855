// ff_quant.cuh — int8 quantisers, int8 transpose and column sums (HBM-bound kernels).
//
// Quantiser math (fireflykernels.py:96-104, same as bitLinear.py:15-27):
//   s = max(absmax, eps) / 127  (fp32, IEEE divide)
//   q = clamp(rint(v / s), -127, 127)  (IEEE divide, round half to even)
// Integer codes are bit-exact with the reference's torch CPU path.
#pragma once
#include <type_traits>

#include "ff_common.cuh"

namespace ff {

// 8 consecutive input elements held in their storage format (16 B for 2-byte types,
// 32 B for fp32): loads are issued first, conversion happens when values are used.
template <int DT>
struct Raw8;
template <>
struct Raw8<FF_DTYPE_BF16> {
  uint4 w;
  __device__ __forceinline__ void load(const __nv_bfloat16* p) { w = __ldg(reinterpret_cast<const uint4*>(p)); }
  __device__ __forceinline__ void from_local(const __nv_bfloat16* p) { w = *reinterpret_cast<const uint4*>(p); }
  __device__ __forceinline__ void zero() { w = make_uint4(0u, 0u, 0u, 0u); }
  __device__ __forceinline__ float get(int j) const {
    const uint32_t x = j < 2 ? w.x : (j < 4 ? w.y : (j < 6 ? w.z : w.w));
    return __uint_as_float((j & 1) ? (x & 0xFFFF0000u) : (x << 16));
  }
  __device__ __forceinline__ uint32_t word(int p) const {  // elements 2p (low half), 2p+1
    return p == 0 ? w.x : (p == 1 ? w.y : (p == 2 ? w.z : w.w));
  }
  __device__ __forceinline__ f2 pair(int p) const {
    const uint32_t x = word(p);
    return mk2(__uint_as_float(x << 16), __uint_as_float(x & 0xFFFF0000u));
  }
};
template <>
struct Raw8<FF_DTYPE_F16> {
  uint4 w;
  __device__ __forceinline__ void load(const __half* p) { w = __ldg(reinterpret_cast<const uint4*>(p)); }
  __device__ __forceinline__ void from_local(const __half* p) { w = *reinterpret_cast<const uint4*>(p); }
  __device__ __forceinline__ void zero() { w = make_uint4(0u, 0u, 0u, 0u); }
  __device__ __forceinline__ float get(int j) const {
    const uint32_t x = j < 2 ? w.x : (j < 4 ? w.y : (j < 6 ? w.z : w.w));
    return __half2float(__ushort_as_half((unsigned short)((j & 1) ? (x >> 16) : (x & 0xFFFFu))));
  }
  __device__ __forceinline__ f2 pair(int p) const { return mk2(get(2 * p), get(2 * p + 1)); }
};
template <>
struct Raw8<FF_DTYPE_F32> {
  float4 a, b;
  __device__ __forceinline__ void load(const float* p) {
    a = __ldg(reinterpret_cast<const float4*>(p));
    b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  }
  __device__ __forceinline__ void from_local(const float* p) {
    a = *reinterpret_cast<const float4*>(p);
    b = *(reinterpret_cast<const float4*>(p) + 1);
  }
  __device__ __forceinline__ void zero() { a = b = make_float4(0.f, 0.f, 0.f, 0.f); }
  __device__ __forceinline__ float get(int j) const {
    const float4& h = j < 4 ? a : b;
    const int k = j & 3;
    return k == 0 ? h.x : (k == 1 ? h.y : (k == 2 ? h.z : h.w));
  }
  __device__ __forceinline__ f2 pair(int p) const { return mk2(get(2 * p), get(2 * p + 1)); }
};

// 8 elements starting at column c of row xr (vector load when allowed, else guarded scalars)
template <int DT>
__device__ __forceinline__ void load_raw8(Raw8<DT>& r, const typename Elem<DT>::T* xr, int64_t c, int64_t cols,
                                          bool vec) {
  if (vec) {
    r.load(xr + c);
  } else {
    // slow path: build the storage-format vector from guarded scalar loads (a local
    // array, read back with generic loads: the non-coherent global path does not apply)
    alignas(16) typename Elem<DT>::T tmp[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) tmp[j] = (c + j < cols) ? xr[c + j] : typename Elem<DT>::T(0.f);
    r.from_local(tmp);
  }
}

// ---------------------------------------------------------------------------
// Element sources of the dual quantiser's absmax pass.  A source turns raw row loads
// into the values of its NOUT column panels; the plain source is the input itself, the
// SwiGLU sources compute the activation (or its gradients) from the GEMM outputs and
// have the pass store them (bf16) for the quantiser pass.  Every source maps all-zero
// raw inputs (rows and columns past the end are loaded as zeros) to the value 0.
// ---------------------------------------------------------------------------
template <int DT>
struct PlainSrc {
  static constexpr int NOUT = 1;
  static constexpr bool kPreloadBoth = true;  // small raw: keep all 8 rows of a thread in flight
  static constexpr bool kStore = false;       // pass A never writes the values back
  static constexpr int kMinBlocks = 2;        // pass A blocks per SM the registers must allow
  static constexpr int kRowsInFlight = 8;     // pass A rows loaded per thread before the math
  static constexpr bool kWords = DT == FF_DTYPE_BF16;  // values available as bf16x2 words
  using T = typename Elem<DT>::T;
  const T* x;
  int64_t ld;
  struct Raw {
    Raw8<DT> v;
    __device__ __forceinline__ void zero() { v.zero(); }
  };
  __device__ __forceinline__ bool vec(int64_t c, int64_t cols) const {
    return (c + 8 <= cols) && ((ld * (int64_t)sizeof(T)) % 16 == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
  }
  __device__ __forceinline__ void load(Raw& r, int64_t row, int64_t c, int64_t cols, bool v) const {
    load_raw8<DT>(r.v, x + row * ld, c, cols, v);
  }
  __device__ __forceinline__ void eval8(const Raw& r, float (&out)[NOUT][8]) const {
#pragma unroll
    for (int j = 0; j < 8; ++j) out[0][j] = r.v.get(j);
  }
  __device__ __forceinline__ void eval_words(const Raw& r, uint32_t (&w)[NOUT][4]) const {
    if constexpr (DT == FF_DTYPE_BF16) {
      w[0][0] = r.v.w.x;
      w[0][1] = r.v.w.y;
      w[0][2] = r.v.w.z;
      w[0][3] = r.v.w.w;
    }
  }
};

// ---------------------------------------------------------------------------
// SwiGLU arithmetic.  torch evaluates, per element x of the gate (a bf16 value, fp32 math):
//   silu(x)        = x / (1 + exp(-x))                         (IEEE divide)
//   sigmoid(x)     = 1 / (1 + exp(-x))                         (IEEE divide)
//   silu_backward  = d * sigmoid * (1 + x * (1 - sigmoid))
// The IEEE divide is a branch around a slow path, which serialises the kernels that
// evaluate it per element.  swiglu_fast computes the same values without branches:
//   den = 1 + expf(-x)                    (the same expf as torch)
//   s   = y + y * (1 - den * y)           y = rcp.approx(den): one Newton-Raphson step
//   q   = q0 + s * (x - den * q0)         q0 = x * s: one residual correction
// (Markstein's correction steps for reciprocal and quotient, "Computation of elementary
// functions on the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990).
// x is a bf16 value, so the inputs form a finite set of 65536 values: swiglu_selftest_kernel
// checks s == RN(1/den) and q == RN(x/den) for every one of them on the running device
// (ff_swiglu_selftest; the Python layer runs it once per device before the first SwiGLU
// call and refuses to continue on a device where it fails).  Inputs outside the range of the fast path (x <= -87: den >= 2^126, where 1/den is
// subnormal and rcp.approx flushes it; x not finite) set `rare` and are recomputed with the
// IEEE operations by the caller.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float rcp_approx_ftz(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
__device__ __forceinline__ uint32_t abs_bf16x2(uint32_t w) { return w & 0x7FFF7FFFu; }
__device__ __forceinline__ uint32_t max_bf16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

struct SwigluMath {
  float den, s, q;  // 1 + exp(-x), RN(1/den), RN(x/den)
};
// x / den has the sign of x (the correction step would turn -0 into +0)
__device__ __forceinline__ float sign_of(float v, float x) { return copysignf(v, x); }
__device__ __forceinline__ SwigluMath swiglu_fast(float x, bool& rare) {
  SwigluMath m;
  m.den = __fadd_rn(1.f, expf(-x));
  const float y = rcp_approx_ftz(m.den);
  m.s = __fmaf_rn(__fmaf_rn(-m.den, y, 1.f), y, y);
  const float q0 = __fmul_rn(x, m.s);
  m.q = sign_of(__fmaf_rn(__fmaf_rn(-m.den, q0, x), m.s, q0), x);
  rare |= !(m.den < 0x1p126f) || !(x < INFINITY);
  return m;
}
// the same on a pair of inputs (f32x2 arithmetic); s and q as pairs
struct SwigluMath2 {
  f2 s, q;
};
__device__ __forceinline__ SwigluMath2 swiglu_fast2(float x0, float x1, bool& rare) {
  const f2 x = mk2(x0, x1), one = splat(1.f);
  const float e0 = expf(-x0), e1 = expf(-x1);
  const f2 e = mk2(e0, e1);
  const f2 nden = sub2(splat(-1.f), e);  // -(1 + e), rounded as 1 + e
  float d0, d1;
  un2(add2(one, e), d0, d1);
  const f2 y = mk2(rcp_approx_ftz(d0), rcp_approx_ftz(d1));
  SwigluMath2 m;
  m.s = fma2(fma2(nden, y, one), y, y);
  const f2 q0 = mul2(x, m.s);
  float q0a, q0b;
  un2(fma2(fma2(nden, q0, x), m.s, q0), q0a, q0b);
  m.q = mk2(sign_of(q0a, x0), sign_of(q0b, x1));
  rare |= !(d0 < 0x1p126f) || !(d1 < 0x1p126f) || !(x0 < INFINITY) || !(x1 < INFINITY);
  return m;
}
// swiglu_fast2 without its range flag, for callers that route inputs with |x| >= 64 (bf16 bit
// patterns with magnitude >= 0x4280, non-finite ones included) to the IEEE path themselves: every
// x with |x| < 64 lies inside the fast path's range (1 + exp(-x) < 2^93)
__device__ __forceinline__ SwigluMath2 swiglu_fast2_in_range(float x0, float x1) {
  const f2 x = mk2(x0, x1), one = splat(1.f);
  const f2 e = mk2(expf(-x0), expf(-x1));
  const f2 nden = sub2(splat(-1.f), e);
  float d0, d1;
  un2(add2(one, e), d0, d1);
  const f2 y = mk2(rcp_approx_ftz(d0), rcp_approx_ftz(d1));
  SwigluMath2 m;
  m.s = fma2(fma2(nden, y, one), y, y);
  const f2 q0 = mul2(x, m.s);
  float q0a, q0b;
  un2(fma2(fma2(nden, q0, x), m.s, q0), q0a, q0b);
  m.q = mk2(sign_of(q0a, x0), sign_of(q0b, x1));
  return m;
}
// halfwise unsigned maximum of two words of 16-bit halves
__device__ __forceinline__ uint32_t max_u16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.u16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// true if either bf16 half of the packed magnitudes `mag` (sign bits cleared) is >= 64 or not finite
__device__ __forceinline__ bool bf16x2_outside_64(uint32_t mag) {
  return (mag & 0xFFFFu) >= 0x4280u || (mag >> 16) >= 0x4280u;
}
__device__ __forceinline__ SwigluMath swiglu_exact(float x) {
  SwigluMath m;
  m.den = __fadd_rn(1.f, expf(-x));
  m.s = __fdiv_rn(1.f, m.den);
  m.q = __fdiv_rn(x, m.den);
  return m;
}
// h = bf16(bf16(silu(g)) * u)
__device__ __forceinline__ float swiglu_h(const SwigluMath& m, float u) { return bf16r(__fmul_rn(bf16r(m.q), u)); }
// dg = bf16(silu_backward(bf16(dh * u), g)), du = bf16(dh * bf16(silu(g)))
__device__ __forceinline__ float swiglu_dg(const SwigluMath& m, float x, float dh, float u) {
  const float ds = bf16r(__fmul_rn(dh, u));
  return bf16r(__fmul_rn(__fmul_rn(ds, m.s), __fmaf_rn(x, __fsub_rn(1.f, m.s), 1.f)));
}
__device__ __forceinline__ float swiglu_du(const SwigluMath& m, float dh) { return bf16r(__fmul_rn(dh, bf16r(m.q))); }

// The IEEE path for one bf16x2 word of inputs (called only when an input is outside the fast
// path's range; kept out of line so that the callers' arrays stay in registers)
__device__ __noinline__ uint32_t swiglu_h_exact_word(uint32_t gw, uint32_t uw) {
  const float h0 = swiglu_h(swiglu_exact(__uint_as_float(gw << 16)), __uint_as_float(uw << 16));
  const float h1 = swiglu_h(swiglu_exact(__uint_as_float(gw & 0xFFFF0000u)), __uint_as_float(uw & 0xFFFF0000u));
  return pack_bf16x2(mk2(h0, h1));
}
__device__ __noinline__ uint2 swiglu_bwd_exact_word(uint32_t gw, uint32_t dw, uint32_t uw) {
  float dg[2], du[2];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const float x = __uint_as_float(k ? (gw & 0xFFFF0000u) : (gw << 16));
    const float d = __uint_as_float(k ? (dw & 0xFFFF0000u) : (dw << 16));
    const float u = __uint_as_float(k ? (uw & 0xFFFF0000u) : (uw << 16));
    const SwigluMath m = swiglu_exact(x);
    dg[k] = swiglu_dg(m, x, d, u);
    du[k] = swiglu_du(m, d);
  }
  return make_uint2(pack_bf16x2(mk2(dg[0], dg[1])), pack_bf16x2(mk2(du[0], du[1])));
}

// every bf16 bit pattern x: fast path (where it applies) against the IEEE operations;
// counts[0] = mismatches, counts[1] = inputs routed to the IEEE path, counts[2] = smallest
// mismatching bf16 bit pattern (0xFFFFFFFF if none)
__global__ void swiglu_selftest_kernel(uint32_t* counts) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= 65536u) return;
  const float x = __uint_as_float(i << 16);
  bool rare = false;
  const SwigluMath f = swiglu_fast(x, rare);
  if (rare) {
    atomicAdd(counts + 1, 1u);
    return;
  }
  const SwigluMath e = swiglu_exact(x);
  if (__float_as_uint(f.s) != __float_as_uint(e.s) || __float_as_uint(f.q) != __float_as_uint(e.q) ||
      __float_as_uint(f.den) != __float_as_uint(e.den)) {
    atomicAdd(counts, 1u);
    atomicMin(counts + 2, i);
  }
}

// h = bf16(bf16(silu(g)) * u): the SwiGLU activation between the gate/up and down projections
struct SwigluSrc {
  static constexpr int NOUT = 1;
  static constexpr bool kPreloadBoth = false;
  static constexpr bool kStore = true;  // pass A writes h (bf16) for pass B
  static constexpr int kMinBlocks = 3;
  static constexpr int kRowsInFlight = 4;
  static constexpr bool kWords = true;
  const __nv_bfloat16* g;
  const __nv_bfloat16* u;
  int64_t ld;
  struct Raw {
    Raw8<FF_DTYPE_BF16> g, u;
    __device__ __forceinline__ void zero() {
      g.zero();
      u.zero();
    }
  };
  __device__ __forceinline__ bool vec(int64_t c, int64_t cols) const {
    return (c + 8 <= cols) && (ld % 8 == 0) && ((reinterpret_cast<uintptr_t>(g) & 15) == 0) &&
           ((reinterpret_cast<uintptr_t>(u) & 15) == 0);
  }
  __device__ __forceinline__ void load(Raw& r, int64_t row, int64_t c, int64_t cols, bool v) const {
    load_raw8<FF_DTYPE_BF16>(r.g, g + row * ld, c, cols, v);
    load_raw8<FF_DTYPE_BF16>(r.u, u + row * ld, c, cols, v);
  }
  // the 8 values of a raw vector as bf16x2 words: branch-free, then again with the IEEE
  // operations when an input is outside the fast path's range
  __device__ __forceinline__ void eval_words(const Raw& r, uint32_t (&w)[NOUT][4]) const {
    bool rare = false;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const uint32_t gw = r.g.word(p);
      const SwigluMath2 m = swiglu_fast2(__uint_as_float(gw << 16), __uint_as_float(gw & 0xFFFF0000u), rare);
      w[0][p] = pack_bf16x2(mul2(unpack_bf16x2(pack_bf16x2(m.q)), unpack_bf16x2(r.u.word(p))));
    }
    if (__builtin_expect(rare, 0)) {
#pragma unroll
      for (int p = 0; p < 4; ++p) w[0][p] = swiglu_h_exact_word(r.g.word(p), r.u.word(p));
    }
  }
};

// gradients of h = silu(g) * u given dh, as torch's autograd forms them in bf16; the two
// are the column panels [dg | du] of one gradient matrix (gate and up share one projection):
//   panel 0: dg = bf16(silu_backward(bf16(dh * u), g))
//   panel 1: du = bf16(dh * bf16(silu(g)))
struct SwigluBwdSrc {
  static constexpr int NOUT = 2;
  static constexpr bool kPreloadBoth = false;
  static constexpr bool kStore = true;  // pass A writes [dg | du] (bf16) for pass B
  static constexpr int kMinBlocks = 3;
  static constexpr int kRowsInFlight = 2;
  static constexpr bool kWords = true;
  const __nv_bfloat16* dh;  // [rows, ldh]
  const __nv_bfloat16* g;   // [rows, ld]
  const __nv_bfloat16* u;   // [rows, ld]
  int64_t ldh, ld;
  struct Raw {
    Raw8<FF_DTYPE_BF16> dh, g, u;
    __device__ __forceinline__ void zero() {
      dh.zero();
      g.zero();
      u.zero();
    }
  };
  __device__ __forceinline__ bool vec(int64_t c, int64_t cols) const {
    return (c + 8 <= cols) && (ld % 8 == 0) && (ldh % 8 == 0) && ((reinterpret_cast<uintptr_t>(dh) & 15) == 0) &&
           ((reinterpret_cast<uintptr_t>(g) & 15) == 0) && ((reinterpret_cast<uintptr_t>(u) & 15) == 0);
  }
  __device__ __forceinline__ void load(Raw& r, int64_t row, int64_t c, int64_t cols, bool v) const {
    load_raw8<FF_DTYPE_BF16>(r.dh, dh + row * ldh, c, cols, v);
    load_raw8<FF_DTYPE_BF16>(r.g, g + row * ld, c, cols, v);
    load_raw8<FF_DTYPE_BF16>(r.u, u + row * ld, c, cols, v);
  }
  __device__ __forceinline__ void eval_words(const Raw& r, uint32_t (&w)[NOUT][4]) const {
    bool rare = false;
    const f2 one = splat(1.f);
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const uint32_t gw = r.g.word(p);
      const f2 x = unpack_bf16x2(gw), d = unpack_bf16x2(r.dh.word(p));
      const SwigluMath2 m = swiglu_fast2(__uint_as_float(gw << 16), __uint_as_float(gw & 0xFFFF0000u), rare);
      const f2 ds = unpack_bf16x2(pack_bf16x2(mul2(d, unpack_bf16x2(r.u.word(p)))));
      w[0][p] = pack_bf16x2(mul2(mul2(ds, m.s), fma2(x, sub2(one, m.s), one)));
      w[1][p] = pack_bf16x2(mul2(d, unpack_bf16x2(pack_bf16x2(m.q))));
    }
    if (__builtin_expect(rare, 0)) {
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const uint2 e = swiglu_bwd_exact_word(r.g.word(p), r.dh.word(p), r.u.word(p));
        w[0][p] = e.x;
        w[1][p] = e.y;
      }
    }
  }
};

// ---------------------------------------------------------------------------
// K1: one warp per row.  Pass 1 reads the row for |x*colmul| max, pass 2
// re-reads it (from L1/L2) and writes codes.  VEC path needs 16 B aligned rows.
// ---------------------------------------------------------------------------
template <int DT, bool VEC>
__global__ void __launch_bounds__(256) quant_rows_kernel(
    const typename Elem<DT>::T* __restrict__ x, int64_t rows, int64_t cols, int64_t ldx,
    const float* __restrict__ colmul, float eps, int8_t* __restrict__ q, int64_t ldq,
    float* __restrict__ s) {
  using T = typename Elem<DT>::T;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const T* xr = x + row * ldx;
  int8_t* qr = q + row * ldq;
  float amax = 0.f;
  if constexpr (VEC) {
    const int64_t nvec = cols / 8;
    for (int64_t i = lane; i < nvec; i += 32) {
      float v[8];
      load8<DT>(xr + i * 8, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float t = colmul ? __fmul_rn(v[j], __ldg(colmul + i * 8 + j)) : v[j];
        amax = fmaxf(amax, fabsf(t));
      }
    }
    for (int64_t c = nvec * 8 + lane; c < cols; c += 32) {
      float t = Elem<DT>::to_f32(xr[c]);
      if (colmul) t = __fmul_rn(t, __ldg(colmul + c));
      amax = fmaxf(amax, fabsf(t));
    }
  } else {
    for (int64_t c = lane; c < cols; c += 32) {
      float t = Elem<DT>::to_f32(xr[c]);
      if (colmul) t = __fmul_rn(t, __ldg(colmul + c));
      amax = fmaxf(amax, fabsf(t));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float sc = row_scale(amax, eps);
  const float isc = __frcp_rn(sc);
  if (lane == 0) s[row] = sc;
  if constexpr (VEC) {
    const int64_t nvec = cols / 8;
    for (int64_t i = lane; i < nvec; i += 32) {
      float v[8];
      load8<DT>(xr + i * 8, v);
      int c8[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float t = colmul ? __fmul_rn(v[j], __ldg(colmul + i * 8 + j)) : v[j];
        c8[j] = quant_code_nr(t, sc, isc);
      }
      uint2 w = make_uint2(pack4(c8[0], c8[1], c8[2], c8[3]), pack4(c8[4], c8[5], c8[6], c8[7]));
      *reinterpret_cast<uint2*>(qr + i * 8) = w;
    }
    for (int64_t c = nvec * 8 + lane; c < ldq; c += 32) {
      int code = 0;
      if (c < cols) {
        float t = Elem<DT>::to_f32(xr[c]);
        if (colmul) t = __fmul_rn(t, __ldg(colmul + c));
        code = quant_code_nr(t, sc, isc);
      }
      qr[c] = (int8_t)code;
    }
  } else {
    for (int64_t c = lane; c < ldq; c += 32) {
      int code = 0;
      if (c < cols) {
        float t = Elem<DT>::to_f32(xr[c]);
        if (colmul) t = __fmul_rn(t, __ldg(colmul + c));
        code = quant_code_nr(t, sc, isc);
      }
      qr[c] = (int8_t)code;
    }
  }
}

// ---------------------------------------------------------------------------
// Dual quantiser, pass A: raw absmax per row (of x*colmul) and per column (of x).
// CTA: 256 threads, tile of 128 rows x 1024 columns.  Threads 0-127 take the
// even rows, 128-255 the odd rows; each thread owns 8 columns (16 B of bf16)
// and keeps 4 row loads in flight.  Partial maxima are combined through shared
// memory, then across CTAs with integer atomicMax on the (non-negative) fp32 bit
// patterns, which is exact and order-independent.
// ---------------------------------------------------------------------------
constexpr int kDualARows = 128;
constexpr int kDualAThreads = 256;
constexpr int kDualACols = 1024;

template <class Src>
__global__ void __launch_bounds__(kDualAThreads, Src::kMinBlocks) dual_absmax_kernel(
    Src src, int64_t rows, int64_t cols, const float* __restrict__ colmul, bool want_rows, bool want_cols,
    uint32_t* __restrict__ row_amax, uint32_t* __restrict__ col_amax, __nv_bfloat16* __restrict__ store,
    int64_t lds, float* __restrict__ colsum) {
  constexpr int NO = Src::NOUT;
  constexpr int U = Src::kRowsInFlight;
  constexpr bool W = Src::kWords;
  // colsum (plain bf16 sources only): this CTA's column sums of its 128 rows, fp32, the even
  // rows' sum plus the odd rows' (each in row order), at colsum[blockIdx.y * cols + c]
  constexpr bool kSums = std::is_same_v<Src, PlainSrc<FF_DTYPE_BF16>>;
  __shared__ float red[kDualARows][5];    // per row: 4 warps' partial maxima
  __shared__ float cred[NO][kDualACols];  // odd-row half's column maxima
  __shared__ float csred[kSums ? kDualACols : 1];  // odd-row half's column sums
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int half = tid >> 7, ct = tid & 127;
  const int64_t c0 = (int64_t)blockIdx.x * kDualACols + ct * 8;
  const int64_t r0 = (int64_t)blockIdx.y * kDualARows;
  const bool vec = src.vec(c0, cols);
  const bool vec_store = store && (c0 + 8 <= cols) && (lds % 8 == 0) && (cols % 8 == 0 || NO == 1) &&
                         ((reinterpret_cast<uintptr_t>(store) & 15) == 0);
  // colmul of this thread's 8 columns (pairs), and the column maxima: bf16x2 words of |v|
  // for word sources (the values are bf16, so their maximum is too), fp32 otherwise
  f2 cm2[NO][4];
  float cmax[NO][W ? 1 : 8];
  uint32_t cmaxw[NO][W ? 4 : 1];
#pragma unroll
  for (int o = 0; o < NO; ++o) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int64_t c = c0 + 2 * q;
      cm2[o][q] = mk2((colmul && c < cols) ? __ldg(colmul + o * cols + c) : 1.f,
                      (colmul && c + 1 < cols) ? __ldg(colmul + o * cols + c + 1) : 1.f);
    }
#pragma unroll
    for (int k = 0; k < (W ? 4 : 1); ++k) cmaxw[o][k] = 0u;
#pragma unroll
    for (int j = 0; j < (W ? 1 : 8); ++j) cmax[o][j] = 0.f;
  }
  const int nr = (int)min64(kDualARows, rows - r0);
  f2 csum2[4] = {splat(0.f), splat(0.f), splat(0.f), splat(0.f)};
#pragma unroll 1
  for (int i0 = half; i0 < kDualARows; i0 += 2 * U) {
    typename Src::Raw v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = i0 + 2 * u;
      if (i < nr) src.load(v[u], r0 + i, c0, cols, vec);
      else v[u].zero();
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = i0 + 2 * u;
      float rm = 0.f;
      if constexpr (W) {
        uint32_t wv[NO][4];
        src.eval_words(v[u], wv);  // columns past the end were loaded as zeros: value 0
        if constexpr (kSums) {
          if (colsum && i < nr) {
#pragma unroll
            for (int q = 0; q < 4; ++q) csum2[q] = add2(csum2[q], unpack_bf16x2(wv[0][q]));
          }
        }
        uint32_t rmw = 0u;
#pragma unroll
        for (int o = 0; o < NO; ++o)
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t aw = abs_bf16x2(wv[o][q]);
            cmaxw[o][q] = max_bf16x2(cmaxw[o][q], aw);
            if (colmul) {
              float a0, a1;
              un2(mul2(unpack_bf16x2(aw), cm2[o][q]), a0, a1);  // |v| * colmul (colmul >= 0)
              rm = fmaxf(rm, fmaxf(a0, a1));
            } else {
              rmw = max_bf16x2(rmw, aw);
            }
          }
        if (!colmul) rm = fmaxf(__uint_as_float(rmw << 16), __uint_as_float(rmw & 0xFFFF0000u));
        if (Src::kStore && store && i < nr) {  // the values themselves: panel o at column o*cols
#pragma unroll
          for (int o = 0; o < NO; ++o) {
            __nv_bfloat16* dst = store + (r0 + i) * lds + o * cols + c0;
            if (vec_store) {
              *reinterpret_cast<uint4*>(dst) = make_uint4(wv[o][0], wv[o][1], wv[o][2], wv[o][3]);
            } else {
#pragma unroll
              for (int j = 0; j < 8; ++j)
                if (c0 + j < cols)
                  reinterpret_cast<uint16_t*>(dst)[j] = (uint16_t)(wv[o][j >> 1] >> (16 * (j & 1)));
            }
          }
        }
      } else {
        float ev[NO][8];
        src.eval8(v[u], ev);  // columns past the end were loaded as zeros: value 0
#pragma unroll
        for (int o = 0; o < NO; ++o)
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float e = ev[o][j];
            cmax[o][j] = fmaxf(cmax[o][j], fabsf(e));
            float c2a, c2b;
            un2(cm2[o][j >> 1], c2a, c2b);
            rm = fmaxf(rm, fabsf(colmul ? __fmul_rn(e, (j & 1) ? c2b : c2a) : e));
          }
      }
      if (want_rows) {
#pragma unroll
        for (int sh = 16; sh > 0; sh >>= 1) rm = fmaxf(rm, __shfl_xor_sync(0xffffffffu, rm, sh));
        if (lane == 0) red[i][warp & 3] = rm;
      }
    }
  }
  // column maxima of this thread as floats
  float cfin[NO][8];
#pragma unroll
  for (int o = 0; o < NO; ++o)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if constexpr (W) {
        const uint32_t w = cmaxw[o][j >> 1];
        cfin[o][j] = __uint_as_float((j & 1) ? (w & 0xFFFF0000u) : (w << 16));
      } else {
        cfin[o][j] = cmax[o][j];
      }
    }
  if (want_cols && half == 1) {
#pragma unroll
    for (int o = 0; o < NO; ++o)
#pragma unroll
      for (int j = 0; j < 8; ++j) cred[o][ct * 8 + j] = cfin[o][j];
  }
  if constexpr (kSums) {
    if (colsum && half == 1) {
#pragma unroll
      for (int q = 0; q < 4; ++q) un2(csum2[q], csred[ct * 8 + 2 * q], csred[ct * 8 + 2 * q + 1]);
    }
  }
  __syncthreads();
  if constexpr (kSums) {
    if (colsum && half == 0) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float a0, a1;
        un2(add2(csum2[q], mk2(csred[ct * 8 + 2 * q], csred[ct * 8 + 2 * q + 1])), a0, a1);
        if (c0 + 2 * q < cols) colsum[(int64_t)blockIdx.y * cols + c0 + 2 * q] = a0;
        if (c0 + 2 * q + 1 < cols) colsum[(int64_t)blockIdx.y * cols + c0 + 2 * q + 1] = a1;
      }
    }
  }
  if (want_cols && half == 0) {
#pragma unroll
    for (int o = 0; o < NO; ++o)
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float m = fmaxf(cfin[o][j], cred[o][ct * 8 + j]);
        if (c0 + j < cols) atomicMax(col_amax + o * cols + c0 + j, __float_as_uint(m));
      }
  }
  if (want_rows) {
    for (int i = tid; i < nr; i += kDualAThreads) {
      const float m = fmaxf(fmaxf(red[i][0], red[i][1]), fmaxf(red[i][2], red[i][3]));
      atomicMax(row_amax + r0 + i, __float_as_uint(m));
    }
  }
}

// ---------------------------------------------------------------------------
// Dual quantiser, pass B: 128 x 128 tiles.  Each thread owns 4 rows x 8 cols
// (twice).  Row codes go straight to q_rows; column codes are packed 4 rows
// per word into a shared-memory tile and written transposed (q_cols_t[c, r]).
// ---------------------------------------------------------------------------
constexpr int kTile = 128;

template <int DT>
__global__ void __launch_bounds__(256, DT == FF_DTYPE_F32 ? 2 : 3) dual_quant_kernel(
    const typename Elem<DT>::T* __restrict__ x, int64_t rows, int64_t cols, int64_t ldx,
    const float* __restrict__ colmul, float eps, const uint32_t* __restrict__ row_amax,
    const uint32_t* __restrict__ col_amax, int8_t* __restrict__ q_rows, int64_t ldq,
    float* __restrict__ s_rows, int8_t* __restrict__ q_cols_t, int64_t ldqt,
    float* __restrict__ s_cols) {
  using T = typename Elem<DT>::T;
  // [col][row/4] words; word w of column c is stored at (w + c + c/32) mod 32, which
  // keeps both the column-wise writes and the row-wise reads nearly conflict-free
  __shared__ uint32_t tileT[kTile][kTile / 4];
  __shared__ float srow[kTile], scol[kTile], cmul[kTile], isrow[kTile], iscol[kTile];
  const int tid = threadIdx.x;
  const int64_t C0 = (int64_t)blockIdx.x * kTile, R0 = (int64_t)blockIdx.y * kTile;
  const bool do_rows = (q_rows != nullptr), do_cols = (q_cols_t != nullptr);
  if (tid < kTile) {
    const int64_t r = R0 + tid;
    srow[tid] = (do_rows && r < rows) ? row_scale(__uint_as_float(row_amax[r]), eps) : 1.f;
    isrow[tid] = __frcp_rn(srow[tid]);
    if (do_rows && r < rows && blockIdx.x == 0) s_rows[r] = srow[tid];
  } else {
    const int k = tid - kTile;
    const int64_t c = C0 + k;
    scol[k] = (do_cols && c < cols) ? row_scale(__uint_as_float(col_amax[c]), eps) : 1.f;
    iscol[k] = __frcp_rn(scol[k]);
    cmul[k] = (colmul && c < cols) ? __ldg(colmul + c) : 1.f;
    if (do_cols && c < cols && blockIdx.y == 0) s_cols[c] = scol[k];
  }
  __syncthreads();
  const int cg = tid & 15;   // 8-column group
  const int rg = tid >> 4;   // 4-row group (0..15), plus 16 for the second half
  const int cb = cg * 8;
  const int64_t c = C0 + cb;
  const bool vec_ok = (c + 8 <= cols) && ((ldx * (int64_t)sizeof(T)) % 16 == 0) &&
                      ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
  const bool row_store = do_rows && c < ldq;
  // per column pair: colmul, -s_col, 1/s_col (the quantiser math runs on f32x2 pairs)
  f2 cm2[4], nsc2[4], isc2[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    cm2[q] = mk2(cmul[cb + 2 * q], cmul[cb + 2 * q + 1]);
    nsc2[q] = mk2(-scol[cb + 2 * q], -scol[cb + 2 * q + 1]);
    isc2[q] = mk2(iscol[cb + 2 * q], iscol[cb + 2 * q + 1]);
  }
  // issue all eight row loads of this thread (two 4 x 8 micro-tiles) before any math
  Raw8<DT> raw[2][4];
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int rb = (rg + half * 16) * 4;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t r = R0 + rb + i;
      if (r < rows) load_raw8<DT>(raw[half][i], x + r * ldx, c, cols, vec_ok);
      else raw[half][i].zero();
    }
  }
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int rb = (rg + half * 16) * 4;  // first row of this 4x8 micro-tile within the tile
    uint32_t colw[8];  // column j: the codes of rows rb..rb+3, one byte each
    int8_t* qr = q_rows + (R0 + rb) * ldq + c;
#pragma unroll
    for (int i = 0; i < 4; ++i, qr += ldq) {
      const int64_t r = R0 + rb + i;
      uint32_t tw[8];  // magic-number words: low byte = code
      if (do_rows) {
        const f2 nsr = splat(-srow[rb + i]), isr = splat(isrow[rb + i]);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          words2(quant_words_nr2(mul2(raw[half][i].pair(q), cm2[q]), nsr, isr), tw[2 * q], tw[2 * q + 1]);
        if (row_store && r < rows) {
          if (c + 8 <= ldq) {
            *reinterpret_cast<uint2*>(qr) =
                make_uint2(pack_lo4(tw[0], tw[1], tw[2], tw[3]), pack_lo4(tw[4], tw[5], tw[6], tw[7]));
          } else {
#pragma unroll
            for (int j = 0; j < 8; ++j)
              if (c + j < ldq) qr[j] = (int8_t)(tw[j] & 0xFFu);
          }
        }
      }
      if (do_cols) {  // rows past the end hold zeros: code 0
#pragma unroll
        for (int q = 0; q < 4; ++q) words2(quant_words_nr2(raw[half][i].pair(q), nsc2[q], isc2[q]), tw[2 * q], tw[2 * q + 1]);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (i == 0) colw[j] = tw[j];
          else if (i == 1) colw[j] = put_byte<1>(colw[j], tw[j]);
          else if (i == 2) colw[j] = put_byte<2>(colw[j], tw[j]);
          else colw[j] = put_byte<3>(colw[j], tw[j]);
        }
      }
    }
    if (do_cols) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int cc = cb + j;
        tileT[cc][(rb / 4 + cc + (cc >> 5)) & 31] = colw[j];
      }
    }
  }
  if (!do_cols) return;
  __syncthreads();
  // write the transposed tile: 128 column-rows x 128 bytes, 16 B per thread-iteration
  const int chunk = tid & 7;  // 16-byte chunk (4 words) of the 128-row span
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int k = (tid >> 3) + it * 32;  // column within tile
    const int64_t cc = C0 + k;
    const int64_t r = R0 + chunk * 16;
    if (cc < cols && r < ldqt) {
      const int rot = k + (k >> 5);
      uint4 w = make_uint4(tileT[k][(chunk * 4 + 0 + rot) & 31], tileT[k][(chunk * 4 + 1 + rot) & 31],
                           tileT[k][(chunk * 4 + 2 + rot) & 31], tileT[k][(chunk * 4 + 3 + rot) & 31]);
      *reinterpret_cast<uint4*>(q_cols_t + cc * ldqt + r) = w;
    }
  }
}

// ---------------------------------------------------------------------------
// int8 transpose through shared memory, 64 x 64 tiles (32 B-word packing)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) transpose_i8_kernel(const int8_t* __restrict__ src, int64_t rows,
                                                           int64_t cols, int64_t lds, int8_t* __restrict__ dst,
                                                           int64_t ldd) {
  __shared__ int8_t t[64][64 + 4];
  const int64_t R0 = (int64_t)blockIdx.y * 64, C0 = (int64_t)blockIdx.x * 64;
  const int tid = threadIdx.x;
  // load: 64 rows x 64 bytes, 16 bytes (as 4 words) per thread
  {
    const int r = tid >> 2, cb = (tid & 3) * 16;
    const int64_t gr = R0 + r;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int64_t gc = C0 + cb + j;
      t[r][cb + j] = (gr < rows && gc < cols) ? src[gr * lds + gc] : (int8_t)0;
    }
  }
  __syncthreads();
  // store: dst row = source column, 64 bytes per dst row, 16 per thread
  {
    const int k = tid >> 2, rb = (tid & 3) * 16;
    const int64_t gc = C0 + k;  // dst row
    if (gc < cols) {
      alignas(16) int8_t buf[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) buf[j] = t[rb + j][k];
      const int64_t gr = R0 + rb;
      int8_t* d = dst + gc * ldd + gr;
      if (gr + 16 <= ldd && ((reinterpret_cast<uintptr_t>(d) & 15) == 0)) {
        *reinterpret_cast<uint4*>(d) = *reinterpret_cast<uint4*>(buf);
      } else {
        for (int j = 0; j < 16 && gr + j < ldd; ++j) d[j] = buf[j];
      }
    }
  }
}

// ---------------------------------------------------------------------------
// deterministic column sums: stage 1 per 256-row chunk, stage 2 over chunks
// ---------------------------------------------------------------------------
constexpr int kColsumChunk = 256;

__global__ void colsum_stage1(const __nv_bfloat16* __restrict__ x, int64_t rows, int64_t cols, int64_t ldx,
                              float* __restrict__ ws) {
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t ch = blockIdx.y;
  if (c >= cols) return;
  const int64_t r0 = ch * kColsumChunk, r1 = min64(rows, r0 + kColsumChunk);
  float acc = 0.f;
  for (int64_t r = r0; r < r1; ++r) acc += __bfloat162float(x[r * ldx + c]);
  ws[ch * cols + c] = acc;
}

// per column, the chunks' partial sums in a fixed order: warp w of the CTA adds the w-th eighth of
// the chunks in chunk order, then the eight range sums are added in warp order (32 columns per CTA)
constexpr int kColsumS2Cols = 32;
constexpr int kColsumS2Threads = 256;
__global__ void __launch_bounds__(kColsumS2Threads) colsum_stage2(const float* __restrict__ ws, int64_t nchunks,
                                                                 int64_t cols, __nv_bfloat16* __restrict__ out) {
  constexpr int kSlices = kColsumS2Threads / kColsumS2Cols;
  __shared__ float part[kSlices][kColsumS2Cols];
  const int lane = threadIdx.x % kColsumS2Cols, slice = threadIdx.x / kColsumS2Cols;
  const int64_t c = (int64_t)blockIdx.x * kColsumS2Cols + lane;
  const int64_t per = (nchunks + kSlices - 1) / kSlices;
  const int64_t k0 = min64(nchunks, slice * per), k1 = min64(nchunks, k0 + per);
  float acc = 0.f;
  if (c < cols)
    for (int64_t k = k0; k < k1; ++k) acc += ws[k * cols + c];
  part[slice][lane] = acc;
  __syncthreads();
  if (slice == 0 && c < cols) {
    float t = part[0][lane];
#pragma unroll
    for (int s = 1; s < kSlices; ++s) t += part[s][lane];
    out[c] = __float2bfloat16_rn(t);
  }
}

__global__ void update_int8_weight_kernel(int8_t* __restrict__ w, const int32_t* __restrict__ dq, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    // int16 arithmetic as in the reference: int16(w) + int16(dq), then clamp
    const int16_t v = (int16_t)((int16_t)w[i] + (int16_t)dq[i]);
    w[i] = (int8_t)min(127, max(-127, (int)v));
  }
}

}  // namespace ff

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" int ff_quant_rows_i8(const void* x, int dtype, int64_t rows, int64_t cols, int64_t ldx,
                                const float* colmul, float eps, int8_t* q, int64_t ldq, float* s,
                                void* stream) {
  using namespace ff;
  FF_REQUIRE(rows >= 0 && cols >= 1, FF_ERR_INVALID_ARG, "ff_quant_rows_i8: rows=%lld cols=%lld",
             (long long)rows, (long long)cols);
  FF_REQUIRE(ldx >= cols && ldq >= cols, FF_ERR_INVALID_ARG, "ff_quant_rows_i8: bad leading dims");
  FF_REQUIRE(dtype == FF_DTYPE_F32 || dtype == FF_DTYPE_BF16 || dtype == FF_DTYPE_F16, FF_ERR_INVALID_ARG,
             "ff_quant_rows_i8: bad dtype %d", dtype);
  if (rows == 0) return FF_OK;
  FF_REQUIRE(x && q && s, FF_ERR_INVALID_ARG, "ff_quant_rows_i8: null pointer");
  const int es = dtype_size(dtype);
  const bool vec = aligned(x, 16) && ((ldx * es) % 16 == 0) && aligned(q, 8) && (ldq % 8 == 0);
  dim3 grid((unsigned)((rows + 7) / 8)), block(256);
  cudaStream_t st = as_stream(stream);
#define FF_QR(DT)                                                                                     \
  if (vec)                                                                                            \
    quant_rows_kernel<DT, true><<<grid, block, 0, st>>>((const Elem<DT>::T*)x, rows, cols, ldx, colmul, \
                                                        eps, q, ldq, s);                              \
  else                                                                                                \
    quant_rows_kernel<DT, false><<<grid, block, 0, st>>>((const Elem<DT>::T*)x, rows, cols, ldx, colmul, \
                                                         eps, q, ldq, s);
  if (dtype == FF_DTYPE_F32) {
    FF_QR(FF_DTYPE_F32)
  } else if (dtype == FF_DTYPE_BF16) {
    FF_QR(FF_DTYPE_BF16)
  } else {
    FF_QR(FF_DTYPE_F16)
  }
#undef FF_QR
  return check_launch("ff_quant_rows_i8");
}

namespace ff {
// Pass A over one source (absmax_ws: rows + NOUT*cols floats, cleared here); with `store`
// the source's values are also written as bf16, panel o at columns o*cols.. of store.
template <class Src>
int launch_pass_a(const char* name, const Src& src, int64_t rows, int64_t cols, const float* colmul,
                  bool do_rows, bool do_cols, float* absmax_ws, __nv_bfloat16* store, int64_t lds,
                  cudaStream_t st, float* colsum = nullptr) {
  uint32_t* row_amax = reinterpret_cast<uint32_t*>(absmax_ws);
  FF_CUDA_TRY(cudaMemsetAsync(absmax_ws, 0, sizeof(float) * (size_t)(rows + Src::NOUT * cols), st), name);
  dim3 gA((unsigned)((cols + kDualACols - 1) / kDualACols), (unsigned)((rows + kDualARows - 1) / kDualARows));
  FF_REQUIRE(gA.y < 65536, FF_ERR_UNSUPPORTED, "%s: too many rows", name);
  dual_absmax_kernel<Src><<<gA, kDualAThreads, 0, st>>>(src, rows, cols, colmul, do_rows, do_cols, row_amax,
                                                         row_amax + rows, store, lds, colsum);
  return check_launch(name);
}

// Pass B over a matrix x of type DT whose absmax values pass A left in absmax_ws.
template <int DT>
int launch_pass_b(const char* name, const typename Elem<DT>::T* x, int64_t rows, int64_t cols, int64_t ldx,
                  const float* colmul, float eps, int8_t* q_rows, int64_t ldq, float* s_rows, int8_t* q_cols_t,
                  int64_t ldqt, float* s_cols, const float* absmax_ws, cudaStream_t st) {
  const uint32_t* row_amax = reinterpret_cast<const uint32_t*>(absmax_ws);
  const int64_t rspan = q_cols_t ? max64(rows, ldqt) : rows;
  const int64_t cspan = q_rows ? max64(cols, ldq) : cols;
  dim3 gB((unsigned)((cspan + kTile - 1) / kTile), (unsigned)((rspan + kTile - 1) / kTile));
  FF_REQUIRE(gB.y < 65536, FF_ERR_UNSUPPORTED, "%s: too many rows", name);
  dual_quant_kernel<DT><<<gB, 256, 0, st>>>(x, rows, cols, ldx, colmul, eps, row_amax, row_amax + rows, q_rows,
                                            ldq, s_rows, q_cols_t, ldqt, s_cols);
  return check_launch(name);
}

// shared argument checks of the dual quantisers' outputs
inline int check_dual_outputs(const char* name, int64_t rows, int64_t cols, const int8_t* q_rows,
                              int64_t ldq, const float* s_rows, const int8_t* q_cols_t, int64_t ldqt,
                              const float* s_cols, const float* absmax_ws) {
  const bool do_rows = q_rows != nullptr, do_cols = q_cols_t != nullptr;
  FF_REQUIRE(do_rows || do_cols, FF_ERR_INVALID_ARG, "%s: nothing to do", name);
  FF_REQUIRE(absmax_ws, FF_ERR_INVALID_ARG, "%s: null workspace", name);
  if (do_rows) {
    FF_REQUIRE(s_rows && ldq >= cols && ldq % 8 == 0 && aligned(q_rows, 8), FF_ERR_UNSUPPORTED,
               "%s: q_rows needs ldq>=cols, ldq%%8==0, 8-byte alignment", name);
  }
  if (do_cols) {
    FF_REQUIRE(s_cols && ldqt >= rows && ldqt % 16 == 0 && aligned(q_cols_t, 16), FF_ERR_UNSUPPORTED,
               "%s: q_cols_t needs ldqt>=rows, ldqt%%16==0, 16-byte alignment", name);
  }
  return FF_OK;
}
}  // namespace ff

extern "C" int ff_quant_dual_i8(const void* x, int dtype, int64_t rows, int64_t cols, int64_t ldx,
                                const float* row_colmul, float eps, int8_t* q_rows, int64_t ldq,
                                float* s_rows, int8_t* q_cols_t, int64_t ldqt, float* s_cols,
                                float* absmax_ws, void* stream) {
  using namespace ff;
  FF_REQUIRE(rows >= 0 && cols >= 1 && ldx >= cols, FF_ERR_INVALID_ARG,
             "ff_quant_dual_i8: rows=%lld cols=%lld ldx=%lld", (long long)rows, (long long)cols, (long long)ldx);
  FF_REQUIRE(dtype == FF_DTYPE_F32 || dtype == FF_DTYPE_BF16 || dtype == FF_DTYPE_F16, FF_ERR_INVALID_ARG,
             "ff_quant_dual_i8: bad dtype %d", dtype);
  FF_REQUIRE(q_rows || q_cols_t, FF_ERR_INVALID_ARG, "ff_quant_dual_i8: nothing to do");
  if (rows == 0) return FF_OK;
  FF_REQUIRE(x, FF_ERR_INVALID_ARG, "ff_quant_dual_i8: null input");
  const int rc = check_dual_outputs("ff_quant_dual_i8", rows, cols, q_rows, ldq, s_rows, q_cols_t, ldqt,
                                    s_cols, absmax_ws);
  if (rc != FF_OK) return rc;
  cudaStream_t st = as_stream(stream);
#define FF_DQ(DT)                                                                                          \
  {                                                                                                      \
    const auto* xt = (const Elem<DT>::T*)x;                                                              \
    const int ra = launch_pass_a("ff_quant_dual_i8", PlainSrc<DT>{xt, ldx}, rows, cols, row_colmul,      \
                                 q_rows != nullptr, q_cols_t != nullptr, absmax_ws, nullptr, 0, st);     \
    if (ra != FF_OK) return ra;                                                                          \
    return launch_pass_b<DT>("ff_quant_dual_i8", xt, rows, cols, ldx, row_colmul, eps, q_rows, ldq,      \
                             s_rows, q_cols_t, ldqt, s_cols, absmax_ws, st);                             \
  }
  if (dtype == FF_DTYPE_F32) FF_DQ(FF_DTYPE_F32)
  if (dtype == FF_DTYPE_BF16) FF_DQ(FF_DTYPE_BF16)
  FF_DQ(FF_DTYPE_F16)
#undef FF_DQ
}

extern "C" int64_t ff_quant_dual_db_ws_elems(int64_t rows, int64_t cols) {
  const int64_t nch = (rows + ff::kDualARows - 1) / ff::kDualARows;
  return (nch > 0 ? nch : 1) * (cols > 0 ? cols : 1);
}

extern "C" int ff_quant_dual_i8_db(const uint16_t* x, int64_t rows, int64_t cols, int64_t ldx,
                                   const float* row_colmul, float eps, int8_t* q_rows, int64_t ldq,
                                   float* s_rows, int8_t* q_cols_t, int64_t ldqt, float* s_cols,
                                   float* absmax_ws, uint16_t* db, float* db_ws, void* stream) {
  using namespace ff;
  FF_REQUIRE(rows >= 0 && cols >= 1 && ldx >= cols, FF_ERR_INVALID_ARG,
             "ff_quant_dual_i8_db: rows=%lld cols=%lld ldx=%lld", (long long)rows, (long long)cols,
             (long long)ldx);
  FF_REQUIRE(q_rows || q_cols_t, FF_ERR_INVALID_ARG, "ff_quant_dual_i8_db: nothing to do");
  FF_REQUIRE(db && db_ws, FF_ERR_INVALID_ARG, "ff_quant_dual_i8_db: null db or db workspace");
  cudaStream_t st = as_stream(stream);
  if (rows == 0) {
    FF_CUDA_TRY(cudaMemsetAsync(db, 0, sizeof(uint16_t) * cols, st), "ff_quant_dual_i8_db memset");
    return FF_OK;
  }
  FF_REQUIRE(x, FF_ERR_INVALID_ARG, "ff_quant_dual_i8_db: null input");
  int rc = check_dual_outputs("ff_quant_dual_i8_db", rows, cols, q_rows, ldq, s_rows, q_cols_t, ldqt, s_cols,
                              absmax_ws);
  if (rc != FF_OK) return rc;
  const auto* xb = reinterpret_cast<const __nv_bfloat16*>(x);
  rc = launch_pass_a("ff_quant_dual_i8_db", PlainSrc<FF_DTYPE_BF16>{xb, ldx}, rows, cols, row_colmul,
                     q_rows != nullptr, q_cols_t != nullptr, absmax_ws, nullptr, 0, st, db_ws);
  if (rc != FF_OK) return rc;
  const int64_t nch = (rows + kDualARows - 1) / kDualARows;
  const unsigned g2 = (unsigned)((cols + kColsumS2Cols - 1) / kColsumS2Cols);
  colsum_stage2<<<g2, kColsumS2Threads, 0, st>>>(db_ws, nch, cols, reinterpret_cast<__nv_bfloat16*>(db));
  rc = check_launch("ff_quant_dual_i8_db");
  if (rc != FF_OK) return rc;
  return launch_pass_b<FF_DTYPE_BF16>("ff_quant_dual_i8_db", xb, rows, cols, ldx, row_colmul, eps, q_rows, ldq,
                                      s_rows, q_cols_t, ldqt, s_cols, absmax_ws, st);
}

extern "C" int ff_swiglu_quant_i8(const uint16_t* g, const uint16_t* u, int64_t ld, int64_t rows, int64_t cols,
                                  float eps, uint16_t* h, int64_t ldh, int8_t* q_rows, int64_t ldq, float* s_rows,
                                  int8_t* q_cols_t, int64_t ldqt, float* s_cols, float* absmax_ws, void* stream) {
  using namespace ff;
  FF_REQUIRE(rows >= 0 && cols >= 1 && ld >= cols && ldh >= cols, FF_ERR_INVALID_ARG,
             "ff_swiglu_quant_i8: rows=%lld cols=%lld ld=%lld ldh=%lld", (long long)rows, (long long)cols,
             (long long)ld, (long long)ldh);
  FF_REQUIRE(q_rows || q_cols_t, FF_ERR_INVALID_ARG, "ff_swiglu_quant_i8: nothing to do");
  if (rows == 0) return FF_OK;
  FF_REQUIRE(g && u && h, FF_ERR_INVALID_ARG, "ff_swiglu_quant_i8: null input or h");
  int rc = check_dual_outputs("ff_swiglu_quant_i8", rows, cols, q_rows, ldq, s_rows, q_cols_t, ldqt, s_cols,
                              absmax_ws);
  if (rc != FF_OK) return rc;
  cudaStream_t st = as_stream(stream);
  auto* hb = reinterpret_cast<__nv_bfloat16*>(h);
  const SwigluSrc src{reinterpret_cast<const __nv_bfloat16*>(g), reinterpret_cast<const __nv_bfloat16*>(u), ld};
  rc = launch_pass_a("ff_swiglu_quant_i8", src, rows, cols, nullptr, q_rows != nullptr, q_cols_t != nullptr,
                     absmax_ws, hb, ldh, st);
  if (rc != FF_OK) return rc;
  return launch_pass_b<FF_DTYPE_BF16>("ff_swiglu_quant_i8", hb, rows, cols, ldh, nullptr, eps, q_rows, ldq, s_rows,
                                      q_cols_t, ldqt, s_cols, absmax_ws, st);
}

extern "C" int ff_swiglu_bwd_quant_i8(const uint16_t* dh, int64_t ldh, const uint16_t* g, const uint16_t* u,
                                      int64_t ld, int64_t rows, int64_t cols, const float* colmul, float eps,
                                      uint16_t* dgu, int64_t lddgu, int8_t* q_rows, int64_t ldq, float* s_rows,
                                      int8_t* q_cols_t, int64_t ldqt, float* s_cols, float* absmax_ws,
                                      void* stream) {
  using namespace ff;
  FF_REQUIRE(rows >= 0 && cols >= 1 && ld >= cols && ldh >= cols && lddgu >= 2 * cols, FF_ERR_INVALID_ARG,
             "ff_swiglu_bwd_quant_i8: rows=%lld cols=%lld ld=%lld ldh=%lld lddgu=%lld", (long long)rows,
             (long long)cols, (long long)ld, (long long)ldh, (long long)lddgu);
  FF_REQUIRE(cols % 8 == 0, FF_ERR_UNSUPPORTED, "ff_swiglu_bwd_quant_i8: cols=%lld must be a multiple of 8",
             (long long)cols);
  FF_REQUIRE(q_rows || q_cols_t, FF_ERR_INVALID_ARG, "ff_swiglu_bwd_quant_i8: nothing to do");
  if (rows == 0) return FF_OK;
  FF_REQUIRE(dh && g && u && dgu, FF_ERR_INVALID_ARG, "ff_swiglu_bwd_quant_i8: null input or dgu");
  int rc = check_dual_outputs("ff_swiglu_bwd_quant_i8", rows, 2 * cols, q_rows, ldq, s_rows, q_cols_t, ldqt,
                              s_cols, absmax_ws);
  if (rc != FF_OK) return rc;
  cudaStream_t st = as_stream(stream);
  auto* db = reinterpret_cast<__nv_bfloat16*>(dgu);
  const SwigluBwdSrc src{reinterpret_cast<const __nv_bfloat16*>(dh), reinterpret_cast<const __nv_bfloat16*>(g),
                         reinterpret_cast<const __nv_bfloat16*>(u), ldh, ld};
  rc = launch_pass_a("ff_swiglu_bwd_quant_i8", src, rows, cols, colmul, q_rows != nullptr, q_cols_t != nullptr,
                     absmax_ws, db, lddgu, st);
  if (rc != FF_OK) return rc;
  return launch_pass_b<FF_DTYPE_BF16>("ff_swiglu_bwd_quant_i8", db, rows, 2 * cols, lddgu, colmul, eps, q_rows,
                                      ldq, s_rows, q_cols_t, ldqt, s_cols, absmax_ws, st);
}

namespace ff {
__device__ uint32_t g_swiglu_selftest[3];
}

extern "C" int ff_swiglu_selftest(uint32_t* mismatches, uint32_t* ieee_inputs, uint32_t* first_mismatch) {
  using namespace ff;
  FF_REQUIRE(mismatches && ieee_inputs && first_mismatch, FF_ERR_INVALID_ARG, "ff_swiglu_selftest: null pointer");
  const uint32_t zero[3] = {0u, 0u, 0xFFFFFFFFu};
  FF_CUDA_TRY(cudaMemcpyToSymbol(g_swiglu_selftest, zero, sizeof(zero)), "ff_swiglu_selftest");
  uint32_t* counts = nullptr;
  FF_CUDA_TRY(cudaGetSymbolAddress(reinterpret_cast<void**>(&counts), g_swiglu_selftest), "ff_swiglu_selftest");
  swiglu_selftest_kernel<<<256, 256>>>(counts);
  const int rc = check_launch("ff_swiglu_selftest");
  if (rc != FF_OK) return rc;
  uint32_t out[3];
  FF_CUDA_TRY(cudaMemcpyFromSymbol(out, g_swiglu_selftest, sizeof(out)), "ff_swiglu_selftest");
  *mismatches = out[0];
  *ieee_inputs = out[1];
  *first_mismatch = out[2];
  return FF_OK;
}

extern "C" int ff_transpose_i8(const int8_t* src, int64_t rows, int64_t cols, int64_t lds, int8_t* dst,
                               int64_t ldd, void* stream) {
  using namespace ff;
  FF_REQUIRE(rows >= 0 && cols >= 0 && lds >= cols && ldd >= rows, FF_ERR_INVALID_ARG,
             "ff_transpose_i8: bad sizes");
  if (rows == 0 || cols == 0) return FF_OK;
  FF_REQUIRE(src && dst, FF_ERR_INVALID_ARG, "ff_transpose_i8: null pointer");
  const int64_t rspan = max64(rows, ldd);
  dim3 grid((unsigned)((cols + 63) / 64), (unsigned)((rspan + 63) / 64));
  FF_REQUIRE(grid.y < 65536, FF_ERR_UNSUPPORTED, "ff_transpose_i8: too many rows");
  transpose_i8_kernel<<<grid, 256, 0, as_stream(stream)>>>(src, rows, cols, lds, dst, ldd);
  return check_launch("ff_transpose_i8");
}

extern "C" int64_t ff_colsum_ws_elems(int64_t rows, int64_t cols) {
  const int64_t nch = (rows + ff::kColsumChunk - 1) / ff::kColsumChunk;
  return (nch > 0 ? nch : 1) * cols;
}

extern "C" int ff_colsum_bf16(const uint16_t* x, int64_t rows, int64_t cols, int64_t ldx, uint16_t* out,
                              float* ws, void* stream) {
  using namespace ff;
  FF_REQUIRE(rows >= 0 && cols >= 0 && ldx >= cols, FF_ERR_INVALID_ARG, "ff_colsum_bf16: bad sizes");
  if (cols == 0) return FF_OK;
  FF_REQUIRE(out && ws && (x || rows == 0), FF_ERR_INVALID_ARG, "ff_colsum_bf16: null pointer");
  cudaStream_t st = as_stream(stream);
  const int64_t nch = (rows + kColsumChunk - 1) / kColsumChunk;
  if (nch == 0) {
    FF_CUDA_TRY(cudaMemsetAsync(out, 0, sizeof(uint16_t) * cols, st), "ff_colsum_bf16 memset");
    return FF_OK;
  }
  FF_REQUIRE(nch < 65536, FF_ERR_UNSUPPORTED, "ff_colsum_bf16: too many rows");
  dim3 g1((unsigned)((cols + 255) / 256), (unsigned)nch);
  colsum_stage1<<<g1, 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(x), rows, cols, ldx, ws);
  const unsigned g2 = (unsigned)((cols + kColsumS2Cols - 1) / kColsumS2Cols);
  colsum_stage2<<<g2, kColsumS2Threads, 0, st>>>(ws, nch, cols, reinterpret_cast<__nv_bfloat16*>(out));
  return check_launch("ff_colsum_bf16");
}

extern "C" int ff_update_int8_weight(int8_t* w, const int32_t* dq, int64_t n, void* stream) {
  using namespace ff;
  FF_REQUIRE(n >= 0, FF_ERR_INVALID_ARG, "ff_update_int8_weight: n < 0");
  if (n == 0) return FF_OK;
  FF_REQUIRE(w && dq, FF_ERR_INVALID_ARG, "ff_update_int8_weight: null pointer");
  const int64_t blocks = min64((n + 255) / 256, 148 * 16);
  update_int8_weight_kernel<<<(unsigned)blocks, 256, 0, as_stream(stream)>>>(w, dq, n);
  return check_launch("ff_update_int8_weight");
}
