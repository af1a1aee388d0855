// ff_common.cuh — shared helpers of the firefly_b200 C ABI (errors, status word,
// bounded waits, element loads).  Compiled for sm_100a only.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>

#include "../../include/firefly_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ != 1000)
#error "firefly_b200 is built for sm_100a only"
#endif

namespace ff {

// ---------------------------------------------------------------------------
// host-side error reporting
// ---------------------------------------------------------------------------
inline std::string& last_error_storage() {
  static thread_local std::string s;
  return s;
}

inline int set_error(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  last_error_storage() = buf;
  return code;
}

inline int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    return set_error(FF_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  }
  return FF_OK;
}

#define FF_REQUIRE(cond, code, ...)            \
  do {                                         \
    if (!(cond)) return ::ff::set_error(code, __VA_ARGS__); \
  } while (0)

#define FF_CUDA_TRY(expr, what)                                               \
  do {                                                                        \
    cudaError_t _e = (expr);                                                  \
    if (_e != cudaSuccess)                                                    \
      return ::ff::set_error(FF_ERR_CUDA, "%s: %s", what, cudaGetErrorString(_e)); \
  } while (0)

__host__ __device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }
__host__ __device__ __forceinline__ int64_t max64(int64_t a, int64_t b) { return a > b ? a : b; }

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// ---------------------------------------------------------------------------
// device status word (one per device, lives in this library's module)
// ---------------------------------------------------------------------------
__device__ uint32_t g_status;

__device__ __forceinline__ void raise_status(uint32_t bits) { atomicOr(&g_status, bits); }

// ---------------------------------------------------------------------------
// time-bounded waits
// ---------------------------------------------------------------------------
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s: no legitimate wait here comes close

// Limit of the in-kernel waits on another unit's progress (mbarrier phases of TMA copies, MMAs,
// epilogues): kWaitLimitNs unless ff_set_wait_limit_ns lowered it, which a test does to make a
// wait run out.  The drains after an abort keep the fixed kWaitLimitNs, so in-flight copies and
// MMAs always finish before a CTA exits.
__device__ uint64_t g_wait_limit_ns = kWaitLimitNs;
__device__ __forceinline__ uint64_t wait_limit_ns() { return *reinterpret_cast<volatile uint64_t*>(&g_wait_limit_ns); }

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------
// element loads
// ---------------------------------------------------------------------------
template <int DT>
struct Elem;
template <>
struct Elem<FF_DTYPE_F32> {
  using T = float;
  static __device__ __forceinline__ float to_f32(T v) { return v; }
};
template <>
struct Elem<FF_DTYPE_BF16> {
  using T = __nv_bfloat16;
  static __device__ __forceinline__ float to_f32(T v) { return __bfloat162float(v); }
};
template <>
struct Elem<FF_DTYPE_F16> {
  using T = __half;
  static __device__ __forceinline__ float to_f32(T v) { return __half2float(v); }
};

inline int dtype_size(int dt) { return dt == FF_DTYPE_F32 ? 4 : 2; }

// load 8 consecutive elements starting at p as fp32 (16 B aligned for 2-byte types,
// two 16 B loads for fp32)
template <int DT>
__device__ __forceinline__ void load8(const typename Elem<DT>::T* p, float (&v)[8]) {
  if constexpr (DT == FF_DTYPE_F32) {
    float4 a = __ldg(reinterpret_cast<const float4*>(p));
    float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    uint4 a = __ldg(reinterpret_cast<const uint4*>(p));
    const typename Elem<DT>::T* e = reinterpret_cast<const typename Elem<DT>::T*>(&a);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = Elem<DT>::to_f32(e[j]);
  }
}

// clamp(rint(v / s), -127, 127) with an IEEE divide: the quantiser of
// fireflykernels.py:102-103 (torch.round is round-half-even)
__device__ __forceinline__ int quant_code(float v, float s) {
  float y = rintf(__fdiv_rn(v, s));
  y = fminf(fmaxf(y, -127.f), 127.f);
  return (y == y) ? (int)y : 0;
}

// The same code as quant_code(v, s), computed from inv_s = 1/s (round-to-nearest).
// y = v * inv_s is within 1.5 ulp of the IEEE quotient v / s, so rint(y) equals
// rint(v / s) except when y lies within a few ulps of a half-integer; only then is
// the exact division done.  Rounding uses the 1.5*2^23 magic add (round half to
// even on the FMA pipe, no float-to-int conversion unit op).
__device__ __forceinline__ int quant_code_fast(float v, float s, float inv_s) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  float y = fminf(fmaxf(__fmul_rn(v, inv_s), -128.f), 128.f);
  float t = __fadd_rn(y, kMagic);
  const float r = __fsub_rn(t, kMagic);
  const float dist = fabsf(fabsf(__fsub_rn(y, r)) - 0.5f);
  if (dist <= 4.8e-7f * fabsf(y)) {  // near a tie: decide with the correctly rounded quotient
    y = fminf(fmaxf(__fdiv_rn(v, s), -128.f), 128.f);
    t = __fadd_rn(y, kMagic);
  }
  const int code = __float_as_int(t) - 0x4B400000;
  return min(127, max(-127, code));
}

// quant_code(v, s) from inv_s = RN(1/s) without a divide: q0 = RN(v * inv_s), the residual
// v - q0*s is exact in one FMA, and RN(q0 + residual * inv_s) is the correctly rounded
// quotient RN(v / s) (Markstein's division theorem for a correctly rounded reciprocal).
// |v| <= 127 * s is assumed (s computed from the absmax of the values being quantised),
// so |v / s| <= 127 and no clamp is needed; rounding is the 1.5*2^23 magic add.
__device__ __forceinline__ int quant_code_nr(float v, float s, float inv_s) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  const float q0 = __fmul_rn(v, inv_s);
  const float q = __fmaf_rn(__fmaf_rn(-q0, s, v), inv_s, q0);
  return __float_as_int(__fadd_rn(q, kMagic)) - 0x4B400000;
}

// The code of quant_code_bounded without its exact fallback: returns rint(v * inv_s) and
// sets `tie` when the result may differ from rint(v / s) (y within a few ulps of a
// half-integer); the caller then recomputes with quant_code.
__device__ __forceinline__ int quant_code_flagged(float v, float inv_s, bool& tie) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  const float y = __fmul_rn(v, inv_s);
  const float t = __fadd_rn(y, kMagic);
  const float dist = fabsf(fabsf(__fsub_rn(y, __fsub_rn(t, kMagic))) - 0.5f);
  tie |= (dist <= 4.8e-7f * fabsf(y));
  return __float_as_int(t) - 0x4B400000;
}

// quant_code_fast when |v| <= 127 * s is known (s computed from the absmax of the very
// values being quantised): |v / s| <= 127, so no clamp is needed before or after rounding.
__device__ __forceinline__ int quant_code_bounded(float v, float s, float inv_s) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  const float y = __fmul_rn(v, inv_s);
  float t = __fadd_rn(y, kMagic);
  const float dist = fabsf(fabsf(__fsub_rn(y, __fsub_rn(t, kMagic))) - 0.5f);
  if (dist <= 4.8e-7f * fabsf(y)) t = __fadd_rn(__fdiv_rn(v, s), kMagic);
  return __float_as_int(t) - 0x4B400000;
}

__device__ __forceinline__ float row_scale(float absmax, float eps) {
  return __fdiv_rn(fmaxf(absmax, eps), 127.f);
}

__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
  return (uint32_t)(a & 0xff) | ((uint32_t)(b & 0xff) << 8) | ((uint32_t)(c & 0xff) << 16) |
         ((uint32_t)(d & 0xff) << 24);
}

// ---------------------------------------------------------------------------
// packed fp32 pairs: Blackwell's f32x2 add/sub/mul/fma issue two IEEE fp32 ops per
// instruction (for kernels bound by instruction issue, not by the FMA pipe)
// ---------------------------------------------------------------------------
struct f2 {
  uint64_t v;
};
__device__ __forceinline__ f2 mk2(float a, float b) {
  f2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r.v) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ f2 splat(float a) { return mk2(a, a); }
__device__ __forceinline__ void un2(f2 x, float& a, float& b) { asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(x.v)); }
__device__ __forceinline__ f2 add2(f2 a, f2 b) {
  f2 r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v));
  return r;
}
__device__ __forceinline__ f2 add2_rm(f2 a, f2 b) {
  f2 r;
  asm("add.rm.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v));
  return r;
}
__device__ __forceinline__ f2 sub2(f2 a, f2 b) {
  f2 r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v));
  return r;
}
__device__ __forceinline__ f2 mul2(f2 a, f2 b) {
  f2 r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v));
  return r;
}
__device__ __forceinline__ f2 fma2(f2 a, f2 b, f2 c) {
  f2 r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r.v) : "l"(a.v), "l"(b.v), "l"(c.v));
  return r;
}

// bf16x2 words: element 2k in the low half, 2k+1 in the high half
__device__ __forceinline__ uint32_t pack_bf16x2(f2 v) {
  float a, b;
  un2(v, a, b);
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ f2 unpack_bf16x2(uint32_t w) {
  return mk2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
}

// low bytes of four words packed into one word (byte k = low byte of the k-th argument)
__device__ __forceinline__ uint32_t pack_lo4(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}
// word w with its byte k (0..3) replaced by the low byte of t
template <int K>
__device__ __forceinline__ uint32_t put_byte(uint32_t w, uint32_t t) {
  constexpr uint32_t sel = K == 0 ? 0x3214u : K == 1 ? 0x3240u : K == 2 ? 0x3410u : 0x4210u;
  return __byte_perm(w, t, sel);
}
// quant_code_nr on a pair, returning the magic-number words (low byte = the int8 code)
__device__ __forceinline__ f2 quant_words_nr2(f2 v, f2 neg_s, f2 inv_s) {
  const f2 q0 = mul2(v, inv_s);
  return add2(fma2(fma2(q0, neg_s, v), inv_s, q0), splat(12582912.0f));
}
__device__ __forceinline__ void words2(f2 x, uint32_t& a, uint32_t& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=r"(a), "=r"(b) : "l"(x.v));
}

// busy-wait for ns nanoseconds of the global timer
__device__ __forceinline__ void spin_ns(uint64_t ns) {
  const uint64_t t0 = globaltimer_ns();
  while (globaltimer_ns() - t0 < ns) {
  }
}

// ---------------------------------------------------------------------------
// TMA tensor maps (cuTensorMapEncodeTiled through the runtime's driver entry point)
// ---------------------------------------------------------------------------
inline PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// bf16 matrix [rows, cols] (leading dim ld) for TMA boxes of box_cols x box_rows elements
inline int make_map_bf16(CUtensorMap* m, const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_cols,
                         int box_rows, CUtensorMapSwizzle swizzle,
                         CUtensorMapL2promotion promo = CU_TENSOR_MAP_L2_PROMOTION_NONE) {
  auto fn = encode_fn();
  if (!fn) return set_error(FF_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, promo, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(FF_ERR_CUDA, "cuTensorMapEncodeTiled (bf16) failed (%d)", (int)r);
  return FF_OK;
}


}  // namespace ff
