// ff_adamw8_dense.cuh — block-wise 8-bit AdamW for dense (non-BitLinear) parameters.
//
// The reference steps dense parameters with bitsandbytes' AdamW8bit (fireflyoptim.py:83,
// :124): Adam moments kept as 8-bit codes of a "dynamic tree" quantisation map, scaled per
// block by the block's absmax (Dettmers et al., "8-bit Optimizers via Block-wise
// Quantization", ICLR 2022).  This kernel implements that algorithm; the two 256-entry maps
// (signed for m, unsigned for v) are built on the host from the paper's description and
// passed in, sorted ascending.
//
// Per element, in fp32 with every operation rounded once (no contractions):
//   m0 = qs[cm] * am,  v0 = qu[cv] * av                 (decode, block absmax am / av)
//   p  = p * (1 - lr*wd)                                (decoupled weight decay; skipped if wd = 0)
//   m  = b1*m0 + (1-b1)*g,   v = b2*v0 + ((1-b2)*g)*g
//   p  = p - a_t * (m / (sqrt(v) + e_t))               a_t = lr*sqrt(bc2)/bc1, e_t = eps*sqrt(bc2)
// (Adam's bias corrections folded into the step size and epsilon, Kingma & Ba, section 2), then
// per block of kBlock elements the new absmax of |m| and v, and each value's code is the nearest
// map entry to value * (1 / absmax) (ties to the lower code).
//
// One CTA per block (256 threads x 8 consecutive elements, vector loads and stores), grid-stride
// over blocks; the maps sit in shared memory in 8 replicas (bank-conflict-light decode), and the
// nearest code is one read of a table of decision thresholds indexed by the value's exponent
// and top fraction bits (see the threshold buckets below).
#pragma once
#include <cmath>

#include "ff_common.cuh"

namespace ff {
namespace dense {

constexpr int kBlock = 2048;
constexpr int kThreads = 256;
constexpr int kPer = kBlock / kThreads;  // 8 elements per thread

struct Params {
  void* p;
  int p_dtype;  // FF_DTYPE_F32 or FF_DTYPE_BF16
  const void* g;
  int g_dtype;
  uint8_t* m_q;
  float* m_absmax;
  uint8_t* v_q;
  float* v_absmax;
  int64_t n;
  float lr, b1, b2, omb1, omb2, decay, step_size, eps_hat;
  int use_decay;
  const float* qs;
  const float* qu;
};

constexpr int kRep = 8;  // map replicas: entry i of replica r at word i*kRep + r (lanes l, l+8, ... share one)

__device__ __forceinline__ float load_elem(const void* base, int dtype, int64_t i) {
  if (dtype == FF_DTYPE_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[i]);
  return reinterpret_cast<const float*>(base)[i];
}

// 8 consecutive elements (fp32 or bf16) starting at a multiple of 8
__device__ __forceinline__ void load8(const void* base, int dtype, int64_t e0, float (&x)[8]) {
  if (dtype == FF_DTYPE_BF16) {
    const uint4 w = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(base) + e0);
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      x[2 * k] = __uint_as_float(ws[k] << 16);
      x[2 * k + 1] = __uint_as_float(ws[k] & 0xFFFF0000u);
    }
  } else {
    const float4 a = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + e0);
    const float4 b = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + e0 + 4);
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
    x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
  }
}

// largest index i with q[i] <= x (q sorted ascending, q[0] <= x), then the nearer of i, i+1;
// q is read from this lane's replica (qr = table + slot, stride kRep).  The general path, for
// maps the bucket tables below cannot serve.
__device__ __forceinline__ int nearest_code(const float* qr, float x) {
  int lo = 0;
#pragma unroll
  for (int step = 128; step > 0; step >>= 1)
    if (qr[(lo + step) * kRep] <= x) lo += step;
  if (lo < 255 && __fsub_rn(qr[(lo + 1) * kRep], x) < __fsub_rn(x, qr[lo * kRep])) ++lo;
  return lo;
}

// ---- threshold buckets
// Over ascending magnitudes M[0..len) the nearest index of a >= 0 (the comparison of the two
// rounded distances fsub(M[k+1], a) < fsub(a, M[k]), or <= when ties go to the larger
// magnitude) is monotone in a, so it equals the number of thresholds t_k <= a, t_k being the
// smallest float at which the choice between M[k] and M[k+1] flips to M[k+1].  A magnitude
// falls in bucket
//   b = clamp((bits(a) >> 16) - kBucketBias, 0, kBuckets - 1)
// (bucket 0: [0, 2^-25); bucket b >= 1: the floats whose top 16 bits, exponent and 7 fraction
// bits, are b + kBucketBias; the last: 1.0 and up).  When no bucket holds two thresholds, the
// bucket's word is  count | (low 16 bits of the threshold inside it, or 0x10000 for none) << 8
// and the nearest index is  count + [low16(a) >= word >> 8]:  one shared-memory read.  The
// tables are built per CTA from the maps and checked; maps they cannot serve (unsorted,
// asymmetric, more than one threshold in a bucket, values above 1) use the search above.
constexpr int kBuckets = 25 * 128 + 2;
constexpr int kBucketBias = (102 << 7) - 1;
constexpr uint32_t kNoThreshold = 0x10000u;
constexpr int kTables = 3;  // signed map's magnitudes (ties to smaller | larger), unsigned map
constexpr int kSmemBytes = 2 * 256 * kRep * 4 + kTables * kBuckets * 4 + 2 * (kThreads / 32) * 4;

__device__ __forceinline__ float bucket_start(int b) {
  return b == 0 ? 0.f : __uint_as_float((uint32_t)(b + kBucketBias) << 16);
}

// whether a is past the threshold between M[k] = lo and M[k+1] = hi
__device__ __forceinline__ bool takes_upper(float lo, float hi, float a, bool ties_up) {
  const float du = __fsub_rn(hi, a), dl = __fsub_rn(a, lo);
  return ties_up ? du <= dl : du < dl;
}

// nearest index by search over magnitudes read at stride kRep (replica 0)
__device__ int nearest_index_search(const float* m0, int len, float a, bool ties_up) {
  int lo = 0;
  for (int step = 128; step > 0; step >>= 1)
    if (lo + step < len && m0[(lo + step) * kRep] <= a) lo += step;
  if (lo + 1 < len && takes_upper(m0[lo * kRep], m0[(lo + 1) * kRep], a, ties_up)) ++lo;
  return lo;
}

// bucket word of bucket b; *bad set when the bucket cannot be described by one word
__device__ uint32_t bucket_word(const float* m0, int len, bool ties_up, int b, int* bad) {
  const int k = nearest_index_search(m0, len, bucket_start(b), ties_up);
  const int kn = b + 1 < kBuckets ? nearest_index_search(m0, len, bucket_start(b + 1), ties_up) : k;
  uint32_t thr = kNoThreshold;
  if (kn - k > 1 || (kn > k && b == 0)) {
    *bad = 1;
  } else if (kn > k) {  // smallest low16 past the threshold, by bisection
    const float lo = m0[k * kRep], hi = m0[(k + 1) * kRep];
    const uint32_t top = (uint32_t)(b + kBucketBias) << 16;
    int l = -1, h = (int)kNoThreshold;  // takes_upper false at l, true at h
    while (h - l > 1) {
      const int mid = (l + h) >> 1;
      if (takes_upper(lo, hi, __uint_as_float(top | (uint32_t)mid), ties_up)) h = mid;
      else l = mid;
    }
    thr = (uint32_t)h;
  }
  return (uint32_t)k | (thr << 8);
}

__device__ __forceinline__ uint32_t bucket_index(const uint32_t* bt, float a) {
  const uint32_t bits = __float_as_uint(a);
  const uint32_t w = bt[min(max((int)(bits >> 16) - kBucketBias, 0), kBuckets - 1)];
  return (w & 0xFFu) + ((bits & 0xFFFFu) >= (w >> 8) ? 1u : 0u);
}

__global__ void __launch_bounds__(kThreads) adamw8_dense_kernel(Params p) {
  extern __shared__ __align__(16) uint32_t smem[];
  float* qs = reinterpret_cast<float*>(smem);  // [256][kRep]
  float* qu = qs + 256 * kRep;                 // [256][kRep]
  uint32_t* bt = smem + 2 * 256 * kRep;        // [kTables][kBuckets]
  uint32_t(*red)[kThreads / 32] = reinterpret_cast<uint32_t(*)[kThreads / 32]>(bt + kTables * kBuckets);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < 256 * kRep; i += kThreads) {
    qs[i] = p.qs[i / kRep];
    qu[i] = p.qu[i / kRep];
  }
  __syncthreads();
  // tables over the signed map's non-negative half qs[128..255] (ties to the smaller magnitude
  // for x >= 0, to the larger for x < 0: both are ties to the lower code) and the unsigned map
  int bad = 0;
  for (int i = tid; i < kTables * kBuckets; i += kThreads) {
    const int t = i / kBuckets, b = i - t * kBuckets;
    bt[i] = t < 2 ? bucket_word(qs + 128 * kRep, 128, t == 1, b, &bad) : bucket_word(qu, 256, false, b, &bad);
  }
  for (int k = tid; k < 256; k += kThreads) {
    if (k < 128) bad |= qs[(127 - k) * kRep] != -qs[(128 + k) * kRep];
    if (k > 0) bad |= !(qs[(k - 1) * kRep] < qs[k * kRep] || k == 128) || !(qu[(k - 1) * kRep] < qu[k * kRep]);
  }
  if (tid == 0) bad |= (qs[128 * kRep] != 0.f) | (qu[0] != 0.f) | !(qs[255 * kRep] <= 1.f) | !(qu[255 * kRep] <= 1.f);
  const bool fast = !__syncthreads_or(bad);
  const uint32_t* bt_dn = bt;
  const uint32_t* bt_up = bt + kBuckets;
  const uint32_t* bt_u = bt + 2 * kBuckets;
  const float* qsr = qs + (lane & (kRep - 1));
  const float* qur = qu + (lane & (kRep - 1));
  const int64_t nblocks = (p.n + kBlock - 1) / kBlock;
  // one block's inputs for this thread: 8 elements of g and p, their m and v codes, and the
  // block's absmax pair (elements past n get g = p = 0 and the zero codes)
  auto load_block = [&](int64_t blk, float (&g)[kPer], float (&w)[kPer], uint32_t (&cm)[2], uint32_t (&cv)[2],
                        float& am, float& av) {
    const int64_t e0 = blk * kBlock + (int64_t)tid * kPer;
    am = p.m_absmax[blk];
    av = p.v_absmax[blk];
    if (e0 + kPer <= p.n) {  // 16-byte (fp32: 2 x 16-byte) vectors and 8-byte code words
      load8(p.g, p.g_dtype, e0, g);
      load8(p.p, p.p_dtype, e0, w);
      const uint2 a = *reinterpret_cast<const uint2*>(p.m_q + e0), b = *reinterpret_cast<const uint2*>(p.v_q + e0);
      cm[0] = a.x; cm[1] = a.y;
      cv[0] = b.x; cv[1] = b.y;
    } else {
      cm[0] = cm[1] = 0x80808080u;
      cv[0] = cv[1] = 0u;
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        const int64_t i = e0 + j;
        const bool in = i < p.n;
        g[j] = in ? load_elem(p.g, p.g_dtype, i) : 0.f;
        w[j] = in ? load_elem(p.p, p.p_dtype, i) : 0.f;
        if (in) {
          const int sh = 8 * (j & 3);
          cm[j >> 2] = (cm[j >> 2] & ~(0xFFu << sh)) | ((uint32_t)p.m_q[i] << sh);
          cv[j >> 2] = (cv[j >> 2] & ~(0xFFu << sh)) | ((uint32_t)p.v_q[i] << sh);
        }
      }
    }
  };
  // software pipeline: the next block's loads are in flight while this one is computed
  float g[kPer], w[kPer], am = 0.f, av = 0.f;
  uint32_t cm[2] = {0u, 0u}, cv[2] = {0u, 0u};
  if ((int64_t)blockIdx.x < nblocks) load_block(blockIdx.x, g, w, cm, cv, am, av);
  for (int64_t blk = blockIdx.x; blk < nblocks; blk += gridDim.x) {
    const int64_t e0 = blk * kBlock + (int64_t)tid * kPer;
    const bool full = e0 + kPer <= p.n;
    float gn[kPer], wn[kPer], amn = 0.f, avn = 0.f;
    uint32_t cmn[2] = {0u, 0u}, cvn[2] = {0u, 0u};
    if (blk + gridDim.x < nblocks) load_block(blk + gridDim.x, gn, wn, cmn, cvn, amn, avn);
    float m[kPer], v[kPer];
    float mx_m = 0.f, mx_v = 0.f;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const uint32_t c_m = (cm[j >> 2] >> (8 * (j & 3))) & 0xFFu, c_v = (cv[j >> 2] >> (8 * (j & 3))) & 0xFFu;
      const float m0 = __fmul_rn(qsr[c_m * kRep], am), v0 = __fmul_rn(qur[c_v * kRep], av);
      if (p.use_decay) w[j] = __fmul_rn(w[j], p.decay);
      m[j] = __fadd_rn(__fmul_rn(p.b1, m0), __fmul_rn(p.omb1, g[j]));
      v[j] = __fadd_rn(__fmul_rn(p.b2, v0), __fmul_rn(__fmul_rn(p.omb2, g[j]), g[j]));
      const float den = __fadd_rn(__fsqrt_rn(v[j]), p.eps_hat);
      w[j] = __fsub_rn(w[j], __fmul_rn(p.step_size, __fdiv_rn(m[j], den)));
      mx_m = fmaxf(mx_m, fabsf(m[j]));  // elements past n have g = 0 and zero codes: m = v = 0
      mx_v = fmaxf(mx_v, fabsf(v[j]));
    }
    // block maxima (non-negative floats order like their bit patterns)
    const uint32_t wm = __reduce_max_sync(0xffffffffu, __float_as_uint(mx_m));
    const uint32_t wv = __reduce_max_sync(0xffffffffu, __float_as_uint(mx_v));
    if (lane == 0) {
      red[0][warp] = wm;
      red[1][warp] = wv;
    }
    __syncthreads();
    uint32_t bm = 0u, bv = 0u;
#pragma unroll
    for (int k = 0; k < kThreads / 32; ++k) {
      bm = max(bm, red[0][k]);
      bv = max(bv, red[1][k]);
    }
    __syncthreads();  // red is rewritten by the next block
    // an all-zero block keeps absmax 0 (its values all decode from the zero code)
    const float nam = __uint_as_float(bm), nav = __uint_as_float(bv);
    const float im = nam > 0.f ? __frcp_rn(nam) : 1.f, iv = nav > 0.f ? __frcp_rn(nav) : 1.f;
    uint32_t om[2] = {0u, 0u}, ov[2] = {0u, 0u};
    // |m| * (1/absmax) can exceed 1 by an ulp: both searches then return the code of 1.0
    if (fast) {
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        // signed: index k of |x| among the magnitudes -> code 128 + k, or 127 - k for x < 0;
        // unsigned: code k
        const float x = __fmul_rn(m[j], im);
        const bool neg = x < 0.f;
        const uint32_t k = bucket_index(neg ? bt_up : bt_dn, fabsf(x));
        om[j >> 2] |= (neg ? 127u - k : 128u + k) << (8 * (j & 3));
        ov[j >> 2] |= bucket_index(bt_u, __fmul_rn(v[j], iv)) << (8 * (j & 3));
      }
    } else {
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        om[j >> 2] |= (uint32_t)nearest_code(qsr, __fmul_rn(m[j], im)) << (8 * (j & 3));
        ov[j >> 2] |= (uint32_t)nearest_code(qur, __fmul_rn(v[j], iv)) << (8 * (j & 3));
      }
    }
    if (full) {
      *reinterpret_cast<uint2*>(p.m_q + e0) = make_uint2(om[0], om[1]);
      *reinterpret_cast<uint2*>(p.v_q + e0) = make_uint2(ov[0], ov[1]);
      if (p.p_dtype == FF_DTYPE_BF16) {
        uint32_t o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const __nv_bfloat162 h = __floats2bfloat162_rn(w[2 * k], w[2 * k + 1]);
          o[k] = *reinterpret_cast<const uint32_t*>(&h);
        }
        *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.p) + e0) = make_uint4(o[0], o[1], o[2], o[3]);
      } else {
        float* pw = reinterpret_cast<float*>(p.p) + e0;
        *reinterpret_cast<float4*>(pw) = make_float4(w[0], w[1], w[2], w[3]);
        *reinterpret_cast<float4*>(pw + 4) = make_float4(w[4], w[5], w[6], w[7]);
      }
    } else {
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        const int64_t i = e0 + j;
        if (i < p.n) {
          p.m_q[i] = (uint8_t)(om[j >> 2] >> (8 * (j & 3)));
          p.v_q[i] = (uint8_t)(ov[j >> 2] >> (8 * (j & 3)));
          if (p.p_dtype == FF_DTYPE_BF16) reinterpret_cast<__nv_bfloat16*>(p.p)[i] = __float2bfloat16_rn(w[j]);
          else reinterpret_cast<float*>(p.p)[i] = w[j];
        }
      }
    }
    if (tid == 0) {
      p.m_absmax[blk] = nam;
      p.v_absmax[blk] = nav;
    }
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      g[j] = gn[j];
      w[j] = wn[j];
    }
    cm[0] = cmn[0]; cm[1] = cmn[1];
    cv[0] = cvn[0]; cv[1] = cvn[1];
    am = amn;
    av = avn;
  }
}

// ---------------------------------------------------------------------------
// fp32-moment AdamW of many small parameters in one launch (the parameters below the 8-bit
// size threshold: norm scales, biases).  The same per-element chain as above without the
// 8-bit codes: the moments are read and written as fp32.  Up to kMultiMax tensors per launch,
// their descriptors passed by value; CTA b works on chunk b - chunk0[t] of tensor t.
// ---------------------------------------------------------------------------
constexpr int kMultiMax = 64;
constexpr int kMultiChunk = 4096;
constexpr int kMultiThreads = 256;

struct MultiParams {
  FfAdamw32Tensor t[kMultiMax];
  int32_t chunk0[kMultiMax + 1];  // first CTA of each tensor; chunk0[count] = the grid size
  int32_t count;
  int32_t use_decay;
  float decay, b1, omb1, b2, omb2;
};
static_assert(sizeof(MultiParams) <= 4096, "kernel parameters of the multi-tensor AdamW");

__global__ void __launch_bounds__(kMultiThreads) adamw32_multi_kernel(const __grid_constant__ MultiParams p) {
  const int b = (int)blockIdx.x;
  int lo = 0, hi = p.count - 1;  // the last tensor whose first CTA is <= b
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (p.chunk0[mid] <= b) lo = mid;
    else hi = mid - 1;
  }
  const FfAdamw32Tensor& d = p.t[lo];
  const int64_t i0 = (int64_t)(b - p.chunk0[lo]) * kMultiChunk;
  const int64_t i1 = min64(i0 + kMultiChunk, d.numel);
  const bool pbf = d.param_dtype == FF_DTYPE_BF16, gbf = d.grad_dtype == FF_DTYPE_BF16;
  for (int64_t i = i0 + threadIdx.x; i < i1; i += kMultiThreads) {
    const float g = gbf ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(d.grad)[i])
                        : reinterpret_cast<const float*>(d.grad)[i];
    float w = pbf ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(d.param)[i])
                  : reinterpret_cast<const float*>(d.param)[i];
    if (p.use_decay) w = __fmul_rn(w, p.decay);
    const float m = __fadd_rn(__fmul_rn(d.exp_avg[i], p.b1), __fmul_rn(g, p.omb1));
    const float v = __fadd_rn(__fmul_rn(d.exp_avg_sq[i], p.b2), __fmul_rn(__fmul_rn(g, p.omb2), g));
    d.exp_avg[i] = m;
    d.exp_avg_sq[i] = v;
    w = __fsub_rn(w, __fmul_rn(__fdiv_rn(m, __fadd_rn(__fsqrt_rn(v), d.eps_term)), d.step_scale));
    if (pbf) reinterpret_cast<__nv_bfloat16*>(d.param)[i] = __float2bfloat16_rn(w);
    else reinterpret_cast<float*>(d.param)[i] = w;
  }
}

}  // namespace dense
}  // namespace ff

extern "C" int ff_adamw32_multi(const FfAdamw32Tensor* tensors, int32_t count, float decay, int32_t use_decay,
                                float beta1, float one_minus_beta1, float beta2, float one_minus_beta2,
                                void* stream) {
  using namespace ff;
  using namespace ff::dense;
  FF_REQUIRE(count >= 0, FF_ERR_INVALID_ARG, "ff_adamw32_multi: count=%d", count);
  if (count == 0) return FF_OK;
  FF_REQUIRE(tensors, FF_ERR_INVALID_ARG, "ff_adamw32_multi: null descriptor array");
  for (int32_t i = 0; i < count; ++i) {
    const FfAdamw32Tensor& d = tensors[i];
    FF_REQUIRE(d.numel >= 0, FF_ERR_INVALID_ARG, "ff_adamw32_multi: tensor %d numel=%lld", i, (long long)d.numel);
    FF_REQUIRE(d.numel == 0 || (d.param && d.grad && d.exp_avg && d.exp_avg_sq), FF_ERR_INVALID_ARG,
               "ff_adamw32_multi: tensor %d has a null pointer", i);
    FF_REQUIRE((d.param_dtype == FF_DTYPE_F32 || d.param_dtype == FF_DTYPE_BF16) &&
                   (d.grad_dtype == FF_DTYPE_F32 || d.grad_dtype == FF_DTYPE_BF16),
               FF_ERR_UNSUPPORTED, "ff_adamw32_multi: tensor %d dtypes %d/%d (fp32 or bf16)", i, d.param_dtype,
               d.grad_dtype);
    FF_REQUIRE(d.numel <= (int64_t)kMultiChunk * 65535, FF_ERR_UNSUPPORTED,
               "ff_adamw32_multi: tensor %d has %lld elements", i, (long long)d.numel);
  }
  cudaStream_t st = as_stream(stream);
  for (int32_t base = 0; base < count; base += kMultiMax) {
    MultiParams prm;
    prm.count = 0;
    int32_t grid = 0;
    for (int32_t i = base; i < count && i < base + kMultiMax; ++i) {
      if (tensors[i].numel == 0) continue;
      prm.t[prm.count] = tensors[i];
      prm.chunk0[prm.count] = grid;
      grid += (int32_t)((tensors[i].numel + kMultiChunk - 1) / kMultiChunk);
      ++prm.count;
    }
    if (prm.count == 0) continue;
    prm.chunk0[prm.count] = grid;
    prm.use_decay = use_decay != 0;
    prm.decay = decay;
    prm.b1 = beta1;
    prm.omb1 = one_minus_beta1;
    prm.b2 = beta2;
    prm.omb2 = one_minus_beta2;
    adamw32_multi_kernel<<<grid, kMultiThreads, 0, st>>>(prm);
    const int rc = check_launch("ff_adamw32_multi");
    if (rc != FF_OK) return rc;
  }
  return FF_OK;
}

extern "C" int ff_adamw8_blockwise(void* p, int p_dtype, const void* g, int g_dtype, uint8_t* m_q, float* m_absmax,
                                   uint8_t* v_q, float* v_absmax, int64_t n, double lr, double beta1, double beta2,
                                   double eps, double weight_decay, int64_t step, const float* qmap_s,
                                   const float* qmap_u, void* stream) {
  using namespace ff;
  using namespace ff::dense;
  FF_REQUIRE(n >= 0 && step >= 1, FF_ERR_INVALID_ARG, "ff_adamw8_blockwise: n=%lld step=%lld", (long long)n,
             (long long)step);
  FF_REQUIRE((p_dtype == FF_DTYPE_F32 || p_dtype == FF_DTYPE_BF16) &&
                 (g_dtype == FF_DTYPE_F32 || g_dtype == FF_DTYPE_BF16),
             FF_ERR_INVALID_ARG, "ff_adamw8_blockwise: parameters and gradients must be fp32 or bf16");
  if (n == 0) return FF_OK;
  FF_REQUIRE(p && g && m_q && m_absmax && v_q && v_absmax && qmap_s && qmap_u, FF_ERR_INVALID_ARG,
             "ff_adamw8_blockwise: null pointer");
  FF_REQUIRE(aligned(p, 16) && aligned(g, 16) && aligned(m_q, 8) && aligned(v_q, 8), FF_ERR_UNSUPPORTED,
             "ff_adamw8_blockwise: p and g need 16-byte, the code arrays 8-byte alignment");
  Params prm;
  prm.p = p;
  prm.p_dtype = p_dtype;
  prm.g = g;
  prm.g_dtype = g_dtype;
  prm.m_q = m_q;
  prm.m_absmax = m_absmax;
  prm.v_q = v_q;
  prm.v_absmax = v_absmax;
  prm.n = n;
  // scalars rounded to fp32 the way torch does for a python float operand
  prm.lr = (float)lr;
  prm.b1 = (float)beta1;
  prm.b2 = (float)beta2;
  prm.omb1 = (float)(1.0 - beta1);
  prm.omb2 = (float)(1.0 - beta2);
  prm.decay = (float)(1.0 - lr * weight_decay);
  prm.use_decay = weight_decay != 0.0;
  const double bc1 = 1.0 - std::pow(beta1, (double)step), bc2 = 1.0 - std::pow(beta2, (double)step);
  FF_REQUIRE(bc1 > 0.0 && bc2 > 0.0, FF_ERR_INVALID_ARG, "ff_adamw8_blockwise: bias corrections must be > 0");
  prm.step_size = (float)(lr * std::sqrt(bc2) / bc1);
  prm.eps_hat = (float)(eps * std::sqrt(bc2));
  prm.qs = qmap_s;
  prm.qu = qmap_u;
  // as many CTAs as are resident at once: each builds its tables once and strides over blocks
  static int resident[64] = {0};
  int dev = 0;
  FF_CUDA_TRY(cudaGetDevice(&dev), "ff_adamw8_blockwise device");
  if (dev < 0 || dev >= 64) return set_error(FF_ERR_UNSUPPORTED, "ff_adamw8_blockwise: device %d", dev);
  if (resident[dev] == 0) {
    FF_CUDA_TRY(cudaFuncSetAttribute(adamw8_dense_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes),
                "ff_adamw8_blockwise smem attribute");
    int per_sm = 0, sms = 0;
    FF_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, adamw8_dense_kernel, kThreads, kSmemBytes),
                "ff_adamw8_blockwise occupancy");
    FF_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "ff_adamw8_blockwise SMs");
    resident[dev] = max(1, per_sm) * sms;
  }
  const int64_t nblocks = (n + kBlock - 1) / kBlock;
  const int grid = (int)min64(nblocks, (int64_t)resident[dev]);
  adamw8_dense_kernel<<<grid, kThreads, kSmemBytes, as_stream(stream)>>>(prm);
  return check_launch("ff_adamw8_blockwise");
}
