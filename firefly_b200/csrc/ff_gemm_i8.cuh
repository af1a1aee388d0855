// ff_gemm_i8.cuh — int8 x int8 -> int32 GEMM on the 5th-generation tensor cores.
//
//   acc[m, n] = sum_k A[m, k] * B[n, k]      (A: M x K, B: N x K, both K-contiguous)
//   D[m, n]   = epilogue(acc)                (raw s32, or scaled fp32 / bf16 / bf16 add)
//
// Persistent, warp-specialised kernel, one CTA per SM:
//   warp 0      TMA producer: 128 x 128 B tile of A and 256 x 128 B tile of B per
//               stage into 128B-swizzled shared memory (4 stages, no multicast)
//   warp 1      allocates 512 TMEM columns (two 128 x 256 s32 accumulators) and
//               issues tcgen05.mma.cta_group::1.kind::i8 (M=128, N=256, K=32)
//   warps 2..5  epilogue: tcgen05.ld 32 columns at a time, scale by the
//               row/column fp32 scales (+bias), convert and store
// The two accumulators let the epilogue of tile i overlap the MMAs of tile i+1.
//
// Every mbarrier wait is bounded by a time limit.  A wait that expires sets
// FF_DEVICE_TIMEOUT in the device status word and an abort flag in shared
// memory; all roles then leave their loops, in-flight TMA loads and MMAs are
// drained with bounded waits, and TMEM is released before the CTA exits.
#pragma once
#include <cudaTypedefs.h>

#include "ff_common.cuh"

namespace ff {
namespace gemm {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 128;  // bytes = int8 elements per stage along K (one 128 B swizzle row)
constexpr int UMMA_K = 32;
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK;  // 16 KiB
constexpr int B_BYTES = BN * BK;  // 32 KiB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int ACC_STAGES = 2;
constexpr int TMEM_COLS = 512;
constexpr int NUM_THREADS = 192;
#ifndef FF_GROUP_M
#define FF_GROUP_M 16
#endif
constexpr int GROUP_M = FF_GROUP_M;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align slack*/ + 256 /*barriers*/;

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ uint32_t mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok;
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int32_t x, int32_t y,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// TMA tile store shared -> global (bulk-group completion); the box is clipped at the tensor's bounds
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// wait until at most one committed bulk group still reads shared memory
__device__ __forceinline__ void bulk_wait_read_1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// make this thread's generic-proxy shared-memory writes visible to the async (TMA) proxy
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void tc_mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor: K-major, 128 B swizzle, 8-row core-matrix
// groups 1024 B apart (SBO), LBO unused for swizzled K-major (encoded 1),
// descriptor version 1 (bits 46-47), layout SWIZZLE_128B = 2 (bits 61-63).
__device__ __forceinline__ uint64_t smem_desc_k_sw128(uint32_t saddr) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Shared-memory matrix descriptor of an MN-major operand tile in 128 B swizzle: each k row
// holds 128 bytes of N, 8-row groups 1024 B apart (SBO), 128-column N chunks `lbo` bytes apart.
__device__ __forceinline__ uint64_t smem_desc_mn_sw128(uint32_t saddr, uint32_t lbo) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor, kind::i8: D s32 (bits 4-5 = 2), A and B signed int8
// (bits 7-9 = 1, bits 10-12 = 1), both K-major, N >> 3 at bits 17-22, M >> 4 at bits 24-28.
__host__ __device__ constexpr uint32_t idesc_i8(int m, int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// ---------------------------------------------------------------------------
// bounded waits
// ---------------------------------------------------------------------------
__device__ __forceinline__ bool wait_bar(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns(), limit = wait_limit_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > limit) {
      *abort_flag = 1;
      raise_status(FF_DEVICE_TIMEOUT);
      return false;
    }
  }
}

// drain wait used after an abort: ignores the abort flag, still time-bounded
__device__ __forceinline__ void drain_bar(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      raise_status(FF_DEVICE_TIMEOUT);
      return;
    }
  }
}

// ---------------------------------------------------------------------------
// tile order: groups of GROUP_M row-tiles walked column by column (L2 reuse of B)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int& tm, int& tn) {
  const int group = GROUP_M * tiles_n;
  const int g = t / group;
  const int first_m = g * GROUP_M;
  const int gsz = min(tiles_m - first_m, GROUP_M);
  const int r = t - g * group;
  tm = first_m + r % gsz;
  tn = r / gsz;
}

struct EpiParams {
  const float* scale_a;
  const float* scale_b;
  const float* bias;
  void* D;
  int64_t ldd;
  int64_t M, N;
  int vec;        // 16-byte vector stores allowed
  int tma_store;  // bf16 output written by TMA tile stores from shared memory (2-CTA kernel)
  // SwiGLU forward epilogue only: h = silu(g) * u (bf16, leading dim ldh), F features,
  // row / column absmax of h (float bits, atomicMax)
  __nv_bfloat16* h;
  int64_t ldh;
  int64_t F;
  uint32_t* row_amax;
  uint32_t* col_amax;
  // SwiGLU backward epilogue only: the saved gate/up output gu = [g | u] (bf16, leading dim
  // ldg_in) and the column multipliers of the [dg | du] row quantiser (fp32 [2F], or null)
  const __nv_bfloat16* g_in;
  int64_t ldg_in;
  const float* colmul;
  // GELU epilogues: the contraction variant of the GELU arithmetic (ff_gelu.cuh)
  int act_variant;
};

// Epilogue kind of the gate/up GEMM of a SwiGLU block (not an FF_OUT_* value): the CTA
// pair's 256 tile columns are 128 gate features and the same 128 up features; the
// epilogue writes g and u (bf16, as FF_OUT_BF16 would) and h = silu(g) * u with the row
// and column absmax of h, i.e. the first pass of the dual quantiser of h.
constexpr int kOutSwigluFwd = 16;
constexpr int kSwigluFeat = 128;  // features per tile
// Epilogue kind of the GEMM dh = dY * W_down of a SwiGLU block's backward: from the dh tile
// and the saved g and u it forms the gradient [dg | du] of gu (bf16), writes it, and folds it
// into the row maxima (with column multipliers) and column maxima: the first pass of the dual
// quantiser of [dg | du].  dh itself is not written.
constexpr int kOutSwigluBwd = 17;
__host__ __device__ constexpr bool is_swiglu(int out) { return out == kOutSwigluFwd || out == kOutSwigluBwd; }
// The ring epilogues (SwiGLU backward: g and u in, dg and du out; GELU backward: u in, du out) run
// kSwbWpq warps per TMEM lane quarter; the tile's 256 features are 16 chunks of kSwbChunk, and warp
// e of a quarter takes chunks e, e + kSwbWpq, ...  The inputs pass through shared memory: per
// epilogue warp a ring of kSwbBufs buffers, each one chunk of the warp's 32 rows of every input
// array, loaded by TMA (32 x 32 B boxes, 32-byte swizzle: the 16-byte half k of row r sits at half
// k ^ ((r >> 2) & 1), so the lanes' row reads and writes hit distinct banks).  The outputs are
// written over the inputs in the same buffer and leave by TMA stores from there; a buffer is loaded
// again once its stores have read it, kSwbBufs - 1 chunks ahead of its use.
constexpr int kSwbChunk = 16;
#ifndef FF_SWB_WPQ
#define FF_SWB_WPQ 3
#endif
#ifndef FF_SWB_BUFS
#define FF_SWB_BUFS 3
#endif
constexpr int kSwbWpq = FF_SWB_WPQ;
constexpr int kSwbWarps = 4 * kSwbWpq;
constexpr int kSwbBufs = FF_SWB_BUFS;
constexpr int kSwbBoxBytes = 32 * kSwbChunk * 2;  // 32 rows x 16 bf16
// after the barriers (256 B): per warp one buffer of the column multipliers of the tile's 256
// features for every output array
constexpr uint32_t kSwbCmOff = 256;
// Epilogue kind of the up GEMM of a GELU MLP block: u (bf16, as FF_OUT_BF16 forms it) and
// h = gelu(u) (tanh form) written by TMA, |h| folded into the row and column maxima: the first
// pass of the dual quantiser of h.
constexpr int kOutGeluFwd = 18;
// Epilogue kind of the GEMM dh = dY * W_down of a GELU MLP block's backward: du = dh * gelu'(u)
// from the dh tile and the saved u, written by TMA and folded into the row maxima (with column
// multipliers) and column maxima; dh itself is not written.
constexpr int kOutGeluBwd = 19;
// the activation epilogues run on 8 warps (two per TMEM lane quarter) with staged column operands
__host__ __device__ constexpr bool is_fused_act(int out) { return out >= kOutSwigluFwd && out <= kOutGeluBwd; }
__host__ __device__ constexpr bool is_gelu(int out) { return out == kOutGeluFwd || out == kOutGeluBwd; }
// The GELU epilogues read gelu(u) (bf16 bits) or gelu'(u) (fp32) from a shared-memory table that
// each CTA fills once (with the same arithmetic) for the bf16 inputs with |u| in [2^-16, 16):
// entry i < kGeluTabSpan is +u with bits (kGeluTabExpLo << 7) + i, entry kGeluTabSpan + i is -u.
// Other inputs (rare for activations) take the arithmetic itself.
constexpr int kGeluTabExpLo = 127 - 16;
constexpr int kGeluTabSpan = 20 * 128;
constexpr int kGeluTabEntries = 2 * kGeluTabSpan;
__device__ __forceinline__ uint32_t gelu_tab_bits(int i) {
  return (i >= kGeluTabSpan ? 0x8000u : 0u) | (uint32_t)((i % kGeluTabSpan) + (kGeluTabExpLo << 7));
}
// The wide epilogues run kSwbWpq warps per TMEM lane quarter on interleaved 16-feature chunks:
// the ring epilogues (SwiGLU backward, GELU backward, whose inputs come through the rings) and the
// GELU forward one (no inputs: u and h leave through two staging buffers per warp).  Layout after
// the pipeline stages: barriers (256 B), the warps' column parameters, the buffers (256-byte
// aligned for the swizzle), the rings' barriers, then the GELU table (gelu' or gelu).
__host__ __device__ constexpr bool is_ring(int out) { return out == kOutSwigluBwd || out == kOutGeluBwd; }
__host__ __device__ constexpr bool is_wide(int out) { return is_ring(out) || out == kOutGeluFwd; }
__host__ __device__ constexpr int ring_arrays(int out) { return out == kOutGeluBwd ? 1 : 2; }  // boxes per chunk
__host__ __device__ constexpr int ring_bufs(int out) { return out == kOutGeluFwd ? 2 : kSwbBufs; }
__host__ __device__ constexpr int ring_buf_bytes(int out) { return ring_arrays(out) * kSwbBoxBytes; }
// per warp: two 256-feature arrays (SwiGLU: gate and up multipliers; GELU forward: column scales
// and bias) or one (GELU backward: the multipliers)
__host__ __device__ constexpr uint32_t ring_cm_bytes(int out) { return (uint32_t)ring_arrays(out) * 256u * 4u; }
__host__ __device__ constexpr uint32_t ring_off(int out) { return kSwbCmOff + kSwbWarps * ring_cm_bytes(out); }
__host__ __device__ constexpr uint32_t ring_bar_off(int out) {
  return ring_off(out) + (uint32_t)(kSwbWarps * ring_bufs(out) * ring_buf_bytes(out));
}
__host__ __device__ constexpr uint32_t ring_tab_off(int out) {
  return ring_bar_off(out) + (uint32_t)(kSwbWarps * ring_bufs(out) * 8);
}
__host__ __device__ constexpr uint32_t ring_ctrl_bytes(int out) {
  return ring_tab_off(out) +
         (out == kOutGeluBwd ? (uint32_t)kGeluTabEntries * 4u : out == kOutGeluFwd ? (uint32_t)kGeluTabEntries * 2u : 0u);
}
static_assert(ring_off(kOutSwigluBwd) % 256 == 0 && ring_off(kOutGeluBwd) % 256 == 0 && ring_off(kOutGeluFwd) % 256 == 0,
              "the buffers must be 256-byte aligned for the 32-byte swizzle");

// table entry of a bf16 bit pattern, or -1 outside the table
__device__ __forceinline__ int gelu_tab_index(uint32_t b16) {
  const int t = (int)(b16 & 0x7FFFu) - (kGeluTabExpLo << 7);
  return (unsigned)t < (unsigned)kGeluTabSpan ? t + ((b16 & 0x8000u) ? kGeluTabSpan : 0) : -1;
}
__device__ __forceinline__ uint32_t lds_u16(uint32_t addr) {
  uint16_t v;
  asm("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ float lds_f32(uint32_t addr) {
  float v;
  asm("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
  return v;
}
__device__ __noinline__ uint32_t gelu_fwd_bits_slow(uint32_t b16, int v) {
  return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(gelu::fwd(__uint_as_float(b16 << 16), v)));
}
__device__ __noinline__ float gelu_grad_slow(uint32_t b16, int v) { return gelu::grad(__uint_as_float(b16 << 16), v); }

template <int OUT>
__device__ __forceinline__ void epilogue_chunk(const uint32_t (&acc)[32], int64_t row, int64_t col0,
                                               const EpiParams& p, float sa, int lane) {
  // per-lane column operands, redistributed with shuffles (all lanes take part)
  const int64_t mycol = col0 + lane;
  float sbl = 1.f, bl = 0.f;
  if constexpr (OUT != FF_OUT_S32) {
    if (p.scale_b && mycol < p.N) sbl = __ldg(p.scale_b + mycol);
    if (p.bias && mycol < p.N) bl = __ldg(p.bias + mycol);
  }
  float v[32];
  if constexpr (OUT != FF_OUT_S32) {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      float t = __int2float_rn((int)acc[j]);
      if (p.scale_a) t = __fmul_rn(t, sa);
      const float sb = __shfl_sync(0xffffffffu, sbl, j);
      const float bj = __shfl_sync(0xffffffffu, bl, j);
      if (p.scale_b) t = __fmul_rn(t, sb);
      if (p.bias) t = __fadd_rn(t, bj);
      v[j] = t;
    }
  }
  if (row >= p.M) return;
  const bool full = (col0 + 32 <= p.N) && p.vec;
  if constexpr (OUT == FF_OUT_S32 || OUT == FF_OUT_F32) {
    uint32_t* d = reinterpret_cast<uint32_t*>(p.D) + row * p.ldd + col0;
    if (full) {
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        uint4 w;
        if constexpr (OUT == FF_OUT_S32) {
          w = make_uint4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
        } else {
          w = make_uint4(__float_as_uint(v[j]), __float_as_uint(v[j + 1]), __float_as_uint(v[j + 2]),
                         __float_as_uint(v[j + 3]));
        }
        *reinterpret_cast<uint4*>(d + j) = w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (col0 + j < p.N) {
          if constexpr (OUT == FF_OUT_S32) d[j] = acc[j];
          else d[j] = __float_as_uint(v[j]);
        }
      }
    }
  } else {
    __nv_bfloat16* d = reinterpret_cast<__nv_bfloat16*>(p.D) + row * p.ldd + col0;
    if (full) {
#pragma unroll
      for (int j = 0; j < 32; j += 8) {
        uint4 w;
        if constexpr (OUT == FF_OUT_BF16_ACCUM) {
          uint4 o = *reinterpret_cast<const uint4*>(d + j);
          const __nv_bfloat16* ob = reinterpret_cast<const __nv_bfloat16*>(&o);
          __nv_bfloat16* nb = reinterpret_cast<__nv_bfloat16*>(&w);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float add = __bfloat162float(__float2bfloat16_rn(v[j + e]));
            nb[e] = __float2bfloat16_rn(__fadd_rn(__bfloat162float(ob[e]), add));
          }
        } else {
          __nv_bfloat16* nb = reinterpret_cast<__nv_bfloat16*>(&w);
#pragma unroll
          for (int e = 0; e < 8; ++e) nb[e] = __float2bfloat16_rn(v[j + e]);
        }
        *reinterpret_cast<uint4*>(d + j) = w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (col0 + j < p.N) {
          if constexpr (OUT == FF_OUT_BF16_ACCUM) {
            const float add = __bfloat162float(__float2bfloat16_rn(v[j]));
            d[j] = __float2bfloat16_rn(__fadd_rn(__bfloat162float(d[j]), add));
          } else {
            d[j] = __float2bfloat16_rn(v[j]);
          }
        }
      }
    }
  }
}

// BMN: B is given MN-major (a K x N row-major matrix) instead of K-major (N x K)
// A warp's 32 x 32 bf16 box (lane = row, 16 bf16x2 words per lane) through one of its two
// shared-memory staging buffers and a TMA tile store at (x, y); `n` counts the warp's stores.
// With SWZ the buffers (512-byte aligned) hold the box in the tensor map's 64-byte swizzle:
// 16-byte chunk k of row r sits at chunk k ^ ((r >> 1) & 3), so the 32 lanes' 16-byte stores
// spread over all banks instead of 8 lanes per bank group.
template <bool SWZ = false>
__device__ __forceinline__ void staged_store(const uint32_t (&w)[16], const CUtensorMap* map, int32_t x, int32_t y,
                                             int lane, uint8_t* stage, uint32_t stage_addr, uint32_t& n) {
  const uint32_t b = n & 1u;
  if (n >= 2) {  // this buffer's previous store must have finished reading it
    if (lane == 0) bulk_wait_read_1();
    __syncwarp();
  }
  uint4* dst = reinterpret_cast<uint4*>(stage + b * 2048 + lane * 64);
  const int sw = SWZ ? (lane >> 1) & 3 : 0;
#pragma unroll
  for (int k = 0; k < 4; ++k) dst[k ^ sw] = make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(map, stage_addr + b * 2048, x, y);
    bulk_commit_group();
  }
  ++n;
}

// One 32 x 32 chunk of a bf16 output through shared memory and a TMA tile store: every lane
// (one row of the warp's 32) converts its 32 values exactly as epilogue_chunk does, writes them
// to a staging buffer, and lane 0 stores the box at (col0, row0).  Two staging buffers per warp
// alternate; `n` counts the warp's stores so far.
__device__ __forceinline__ void epilogue_chunk_tma(const uint32_t (&acc)[32], int64_t col0, int64_t row0,
                                                   const EpiParams& p, const CUtensorMap* tmD, float sa, int lane,
                                                   uint8_t* stage, uint32_t stage_addr, uint32_t& n) {
  const int64_t mycol = col0 + lane;
  float sbl = 1.f, bl = 0.f;
  if (p.scale_b && mycol < p.N) sbl = __ldg(p.scale_b + mycol);
  if (p.bias && mycol < p.N) bl = __ldg(p.bias + mycol);
  uint32_t w[16];
#pragma unroll
  for (int q = 0; q < 16; ++q) {
    float t2[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int j = 2 * q + e;
      float t = __int2float_rn((int)acc[j]);
      if (p.scale_a) t = __fmul_rn(t, sa);
      const float sb = __shfl_sync(0xffffffffu, sbl, j);
      const float bj = __shfl_sync(0xffffffffu, bl, j);
      if (p.scale_b) t = __fmul_rn(t, sb);
      if (p.bias) t = __fadd_rn(t, bj);
      t2[e] = t;
    }
    w[q] = pack_bf16x2(mk2(t2[0], t2[1]));
  }
  staged_store<true>(w, tmD, (int32_t)col0, (int32_t)row0, lane, stage, stage_addr, n);
}

// 32 features of the SwiGLU forward epilogue for one row (one thread): accumulators of the
// gate (ag) and up (au) columns -> g, u (bf16, stored at columns fb and F + fb of D), h (stored
// at column fb of h); folds |h| into the row maximum rmax (bf16x2 word) and the column maxima
// (a reduce-scatter over the warp's 32 rows, then one atomicMax per lane).
// `cb` points at this chunk's entries of the warp's staged buffer: gate scales at [0, 32),
// up scales at [64, 96), gate bias at [128, 160), up bias at [192, 224).
__device__ __forceinline__ void swiglu_fwd_chunk(const uint32_t (&ag)[32], const uint32_t (&au)[32], int64_t row,
                                                 int64_t fb, const EpiParams& p, float sa, int lane,
                                                 const float* cb, uint32_t& rmax, const CUtensorMap* tmD,
                                                 const CUtensorMap* tmH, uint8_t* stage, uint32_t stage_addr,
                                                 uint32_t& nst) {
  const bool live = row < p.M;
  float sg[32], su[32], bg[32], bu[32];
#pragma unroll
  for (int j = 0; j < 32; j += 4) {  // shared-memory broadcasts: every lane reads the same values
    const float4 a = *reinterpret_cast<const float4*>(cb + j);
    const float4 b = *reinterpret_cast<const float4*>(cb + 64 + j);
    sg[j] = a.x; sg[j + 1] = a.y; sg[j + 2] = a.z; sg[j + 3] = a.w;
    su[j] = b.x; su[j + 1] = b.y; su[j + 2] = b.z; su[j + 3] = b.w;
    if (p.bias) {
      const float4 c = *reinterpret_cast<const float4*>(cb + 128 + j);
      const float4 d = *reinterpret_cast<const float4*>(cb + 192 + j);
      bg[j] = c.x; bg[j + 1] = c.y; bg[j + 2] = c.z; bg[j + 3] = c.w;
      bu[j] = d.x; bu[j + 1] = d.y; bu[j + 2] = d.z; bu[j + 3] = d.w;
    }
  }
  // g and u exactly as the FF_OUT_BF16 epilogue forms them: ((acc * sa) * sb) (+ bias) -> bf16
  uint32_t wg[16], wu[16], wh[16];
  const f2 sa2 = splat(sa);
#pragma unroll
  for (int q = 0; q < 16; ++q) {
    f2 vg = mul2(mk2(__int2float_rn((int)ag[2 * q]), __int2float_rn((int)ag[2 * q + 1])), sa2);
    f2 vu = mul2(mk2(__int2float_rn((int)au[2 * q]), __int2float_rn((int)au[2 * q + 1])), sa2);
    vg = mul2(vg, mk2(sg[2 * q], sg[2 * q + 1]));
    vu = mul2(vu, mk2(su[2 * q], su[2 * q + 1]));
    if (p.bias) {
      vg = add2(vg, mk2(bg[2 * q], bg[2 * q + 1]));
      vu = add2(vu, mk2(bu[2 * q], bu[2 * q + 1]));
    }
    wg[q] = pack_bf16x2(vg);
    wu[q] = pack_bf16x2(vu);
  }
  // h = bf16(bf16(silu(g)) * u), branch-free, with the IEEE operations for inputs outside the
  // fast path's range
  bool rare = false;
#pragma unroll
  for (int q = 0; q < 16; ++q) {
    const SwigluMath2 m = swiglu_fast2(__uint_as_float(wg[q] << 16), __uint_as_float(wg[q] & 0xFFFF0000u), rare);
    wh[q] = pack_bf16x2(mul2(unpack_bf16x2(pack_bf16x2(m.q)), unpack_bf16x2(wu[q])));
  }
  if (__builtin_expect(rare, 0)) {
#pragma unroll
    for (int q = 0; q < 16; ++q) wh[q] = swiglu_h_exact_word(wg[q], wu[q]);
  }
  // g, u (columns fb and F + fb of gu) and h: TMA tile stores of the warp's 32 rows (clipped at M)
  const int32_t row0 = (int32_t)(row - lane);
  staged_store<true>(wg, tmD, (int32_t)fb, row0, lane, stage, stage_addr, nst);
  staged_store<true>(wu, tmD, (int32_t)(p.F + fb), row0, lane, stage, stage_addr, nst);
  staged_store<true>(wh, tmH, (int32_t)fb, row0, lane, stage, stage_addr, nst);
  // maxima of |h| (rows past M hold no data: excluded)
  uint32_t a[16];
#pragma unroll
  for (int q = 0; q < 16; ++q) {
    a[q] = live ? abs_bf16x2(wh[q]) : 0u;
    rmax = max_bf16x2(rmax, a[q]);
  }
  // reduce-scatter over the 32 lanes: after the rounds lane l holds the maximum of feature fb + l
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const bool up = lane & 16;
    const uint32_t send = up ? a[q] : a[q + 8], keep = up ? a[q + 8] : a[q];
    a[q] = max_bf16x2(keep, __shfl_xor_sync(0xffffffffu, send, 16));
  }
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const bool up = lane & 8;
    const uint32_t send = up ? a[q] : a[q + 4], keep = up ? a[q + 4] : a[q];
    a[q] = max_bf16x2(keep, __shfl_xor_sync(0xffffffffu, send, 8));
  }
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const bool up = lane & 4;
    const uint32_t send = up ? a[q] : a[q + 2], keep = up ? a[q + 2] : a[q];
    a[q] = max_bf16x2(keep, __shfl_xor_sync(0xffffffffu, send, 4));
  }
  {
    const bool up = lane & 2;
    const uint32_t send = up ? a[0] : a[1], keep = up ? a[1] : a[0];
    a[0] = max_bf16x2(keep, __shfl_xor_sync(0xffffffffu, send, 2));
  }
  a[0] = max_bf16x2(a[0], __shfl_xor_sync(0xffffffffu, a[0], 1));  // word (lane >> 1) & 15, all 32 rows
  const uint32_t bits = (lane & 1) ? (a[0] & 0xFFFF0000u) : (a[0] << 16);
  atomicMax(p.col_amax + fb + lane, bits);
}

// reduce-scatter of 16 bf16x2 words (32 features) over the warp's 32 rows: the maximum of
// feature `lane` over all 32 lanes, as float bits
__device__ __forceinline__ uint32_t warp_colmax_bits(uint32_t (&a)[16], int lane) {
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const bool up = lane & 16;
    const uint32_t send = up ? a[q] : a[q + 8], keep = up ? a[q + 8] : a[q];
    a[q] = max_bf16x2(keep, __shfl_xor_sync(0xffffffffu, send, 16));
  }
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const bool up = lane & 8;
    const uint32_t send = up ? a[q] : a[q + 4], keep = up ? a[q + 4] : a[q];
    a[q] = max_bf16x2(keep, __shfl_xor_sync(0xffffffffu, send, 8));
  }
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const bool up = lane & 4;
    const uint32_t send = up ? a[q] : a[q + 2], keep = up ? a[q + 2] : a[q];
    a[q] = max_bf16x2(keep, __shfl_xor_sync(0xffffffffu, send, 4));
  }
  {
    const bool up = lane & 2;
    const uint32_t send = up ? a[0] : a[1], keep = up ? a[1] : a[0];
    a[0] = max_bf16x2(keep, __shfl_xor_sync(0xffffffffu, send, 2));
  }
  a[0] = max_bf16x2(a[0], __shfl_xor_sync(0xffffffffu, a[0], 1));  // word (lane >> 1) & 15, all 32 rows
  return (lane & 1) ? (a[0] & 0xFFFF0000u) : (a[0] << 16);
}

// reduce-scatter of 8 bf16x2 words (16 features) over the warp's 32 rows: the maximum of feature
// 8*b4 + 4*b3 + 2*b2 + b0 over all 32 lanes (b_i = bit i of the lane), as float bits; lanes with
// bit 1 set hold a copy of their neighbour's feature
__device__ __forceinline__ uint32_t warp_colmax16_bits(uint32_t (&a)[8], int lane) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const bool up = lane & 16;
    const uint32_t send = up ? a[q] : a[q + 4], keep = up ? a[q + 4] : a[q];
    a[q] = max_bf16x2(keep, __shfl_xor_sync(0xffffffffu, send, 16));
  }
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const bool up = lane & 8;
    const uint32_t send = up ? a[q] : a[q + 2], keep = up ? a[q + 2] : a[q];
    a[q] = max_bf16x2(keep, __shfl_xor_sync(0xffffffffu, send, 8));
  }
  {
    const bool up = lane & 4;
    const uint32_t send = up ? a[0] : a[1], keep = up ? a[1] : a[0];
    a[0] = max_bf16x2(keep, __shfl_xor_sync(0xffffffffu, send, 4));
  }
  a[0] = max_bf16x2(a[0], __shfl_xor_sync(0xffffffffu, a[0], 2));
  a[0] = max_bf16x2(a[0], __shfl_xor_sync(0xffffffffu, a[0], 1));  // word 4*b4 + 2*b3 + b2, all 32 rows
  return (lane & 1) ? (a[0] & 0xFFFF0000u) : (a[0] << 16);
}
__device__ __forceinline__ int colmax16_feature(int lane) {
  return ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 + (lane & 1);
}

// kSwbChunk (16) features of the SwiGLU backward epilogue for one row (one thread): dh = bf16(acc *
// sa) (as FF_OUT_BF16 forms it) with the row's g and u (from the ring buffer `buf`, shared address
// buf_addr) gives dg = bf16(silu_backward(bf16(dh * u), g)) and du = bf16(dh * bf16(silu(g))); they
// are written over g and u and stored by TMA at columns fb and F + fb of D (lane 0 issues the
// stores as one bulk group).  Folds |dg * colmul|, |du * colmul| into rmax and |dg|, |du| into the
// column maxima.  `cg`, `cu`: this chunk's 16 gate and 16 up column multipliers.
__device__ __forceinline__ void swiglu_bwd_chunk16(const uint32_t (&acc)[16], uint8_t* buf, uint32_t buf_addr,
                                                   int64_t row, int64_t fb, const EpiParams& p, float sa, int lane,
                                                   const float* cg, const float* cu, float& rmax,
                                                   const CUtensorMap* tmD) {
  const int sw = (lane >> 2) & 1;
  uint4* gp = reinterpret_cast<uint4*>(buf + lane * 32);
  uint4* up = reinterpret_cast<uint4*>(buf + kSwbBoxBytes + lane * 32);
  const uint4 g0 = gp[sw], g1 = gp[sw ^ 1], u0 = up[sw], u1 = up[sw ^ 1];
  const uint32_t gw[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
  const uint32_t uw[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
  const f2 sa2 = splat(sa);
  uint32_t dw[8];
#pragma unroll
  for (int q = 0; q < 8; ++q)
    dw[q] = pack_bf16x2(mul2(mk2(__int2float_rn((int)acc[2 * q]), __int2float_rn((int)acc[2 * q + 1])), sa2));
  uint32_t wdg[8], wdu[8];
  uint32_t gmag = 0u;  // halfwise maximum of |g| (bf16 bits)
  const f2 one = splat(1.f);
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const f2 x = unpack_bf16x2(gw[q]), d = unpack_bf16x2(dw[q]);
    gmag = max_u16x2(gmag, abs_bf16x2(gw[q]));
    const SwigluMath2 m = swiglu_fast2_in_range(__uint_as_float(gw[q] << 16), __uint_as_float(gw[q] & 0xFFFF0000u));
    const f2 ds = unpack_bf16x2(pack_bf16x2(mul2(d, unpack_bf16x2(uw[q]))));
    wdg[q] = pack_bf16x2(mul2(mul2(ds, m.s), fma2(x, sub2(one, m.s), one)));
    wdu[q] = pack_bf16x2(mul2(d, unpack_bf16x2(pack_bf16x2(m.q))));
  }
  if (__builtin_expect(bf16x2_outside_64(gmag), 0)) {  // some |g| >= 64: the IEEE path for the chunk
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const uint2 e = swiglu_bwd_exact_word(gw[q], dw[q], uw[q]);
      wdg[q] = e.x;
      wdu[q] = e.y;
    }
  }
  gp[sw] = make_uint4(wdg[0], wdg[1], wdg[2], wdg[3]);
  gp[sw ^ 1] = make_uint4(wdg[4], wdg[5], wdg[6], wdg[7]);
  up[sw] = make_uint4(wdu[0], wdu[1], wdu[2], wdu[3]);
  up[sw ^ 1] = make_uint4(wdu[4], wdu[5], wdu[6], wdu[7]);
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    const int32_t row0 = (int32_t)(row - lane);
    tma_store_2d(tmD, buf_addr, (int32_t)fb, row0);
    tma_store_2d(tmD, buf_addr + kSwbBoxBytes, (int32_t)(p.F + fb), row0);
    bulk_commit_group();
  }
  // rows past M have zero dh, g and u (TMA fills them with zeros), so their dg and du are zeros
  uint32_t ag[8], au[8];
  uint32_t rw = 0u;
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    ag[q] = abs_bf16x2(wdg[q]);
    au[q] = abs_bf16x2(wdu[q]);
    if (p.colmul) {  // |v| * colmul (colmul >= 0) in fp32, as the row quantiser takes it
      float a0, a1, b0, b1;
      un2(mul2(unpack_bf16x2(ag[q]), mk2(cg[2 * q], cg[2 * q + 1])), a0, a1);
      un2(mul2(unpack_bf16x2(au[q]), mk2(cu[2 * q], cu[2 * q + 1])), b0, b1);
      rmax = fmaxf(rmax, fmaxf(fmaxf(a0, a1), fmaxf(b0, b1)));
    } else {
      rw = max_bf16x2(rw, max_bf16x2(ag[q], au[q]));
    }
  }
  if (!p.colmul) rmax = fmaxf(rmax, fmaxf(__uint_as_float(rw << 16), __uint_as_float(rw & 0xFFFF0000u)));
  const uint32_t mg = warp_colmax16_bits(ag, lane), mu = warp_colmax16_bits(au, lane);
  if (!(lane & 2)) {
    const int f = colmax16_feature(lane);
    atomicMax(p.col_amax + fb + f, mg);
    atomicMax(p.col_amax + p.F + fb + f, mu);
  }
}

// kSwbChunk (16) features of the GELU forward epilogue for one row (one thread): u exactly as the
// FF_OUT_BF16 epilogue forms it (((acc * sa) * sb) (+ bias) -> bf16) and h = bf16(gelu(u)) (from the
// shared table at `tab`, the arithmetic itself outside it) are written to the staging buffer `buf`
// (shared address buf_addr: the u box, then the h box, 32-byte swizzle) and stored by TMA at column
// fb of D and H (lane 0 issues both stores as one bulk group); |h| is folded into the row maximum
// rmax (bf16x2 word) and the column maxima.  `sb`, `bb`: this chunk's 16 column scales and biases.
__device__ __forceinline__ void gelu_fwd_chunk16(const uint32_t (&acc)[16], uint8_t* buf, uint32_t buf_addr,
                                                 int64_t row, int64_t fb, const EpiParams& p, float sa, int lane,
                                                 const float* sb, const float* bb, uint32_t tab, uint32_t& rmax,
                                                 const CUtensorMap* tmD, const CUtensorMap* tmH) {
  const bool live = row < p.M;
  uint32_t wu[8], wh[8];
  bool rare = false;
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    // ((acc * sa) * sb) + bias, each step rounded (never contracted), with the missing factors 1 and
    // the missing bias -0 (exact identities)
    float t2[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int j = 2 * q + e;
      t2[e] = __fadd_rn(__fmul_rn(__fmul_rn(__int2float_rn((int)acc[j]), sa), sb[j]), bb[j]);
    }
    wu[q] = pack_bf16x2(mk2(t2[0], t2[1]));
    const int i0 = gelu_tab_index(wu[q] & 0xFFFFu), i1 = gelu_tab_index(wu[q] >> 16);
    rare |= (i0 | i1) < 0;
    wh[q] = lds_u16(tab + 2u * (uint32_t)max(i0, 0)) | (lds_u16(tab + 2u * (uint32_t)max(i1, 0)) << 16);
  }
  if (__builtin_expect(rare, 0)) {  // inputs outside the table: the arithmetic itself
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const uint32_t b0 = wu[q] & 0xFFFFu, b1 = wu[q] >> 16;
      if (gelu_tab_index(b0) < 0) wh[q] = (wh[q] & 0xFFFF0000u) | gelu_fwd_bits_slow(b0, p.act_variant);
      if (gelu_tab_index(b1) < 0) wh[q] = (wh[q] & 0xFFFFu) | (gelu_fwd_bits_slow(b1, p.act_variant) << 16);
    }
  }
  const int sw = (lane >> 2) & 1;
  uint4* ud = reinterpret_cast<uint4*>(buf + lane * 32);
  uint4* hd = reinterpret_cast<uint4*>(buf + kSwbBoxBytes + lane * 32);
  ud[sw] = make_uint4(wu[0], wu[1], wu[2], wu[3]);
  ud[sw ^ 1] = make_uint4(wu[4], wu[5], wu[6], wu[7]);
  hd[sw] = make_uint4(wh[0], wh[1], wh[2], wh[3]);
  hd[sw ^ 1] = make_uint4(wh[4], wh[5], wh[6], wh[7]);
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    const int32_t row0 = (int32_t)(row - lane);
    tma_store_2d(tmD, buf_addr, (int32_t)fb, row0);
    tma_store_2d(tmH, buf_addr + kSwbBoxBytes, (int32_t)fb, row0);
    bulk_commit_group();
  }
  uint32_t a[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    a[q] = live ? abs_bf16x2(wh[q]) : 0u;  // rows past M hold no data (their h is gelu(bias))
    rmax = max_bf16x2(rmax, a[q]);
  }
  const uint32_t m = warp_colmax16_bits(a, lane);
  if (!(lane & 2)) atomicMax(p.col_amax + fb + colmax16_feature(lane), m);
}

// kSwbChunk (16) features of the GELU backward epilogue for one row (one thread): dh = bf16(acc * sa)
// (as FF_OUT_BF16 forms it) and the row's u (from the ring buffer `buf`, shared address buf_addr) give
// du = bf16(dh * gelu'(u)) (gelu' from the shared table at `tab`, the arithmetic itself outside it),
// written over u and stored by TMA at column fb of D (lane 0 issues the store as one bulk group).
// Folds |du * colmul| into rmax and |du| into the column maxima.  `cm`: this chunk's 16 multipliers.
// Rows past M have zero dh and u (TMA fills them with zeros), so their du is zero.
__device__ __forceinline__ void gelu_bwd_chunk16(const uint32_t (&acc)[16], uint8_t* buf, uint32_t buf_addr,
                                                 int64_t row, int64_t fb, const EpiParams& p, float sa, int lane,
                                                 const float* cm, uint32_t tab, float& rmax, const CUtensorMap* tmD) {
  const int sw = (lane >> 2) & 1;
  uint4* up = reinterpret_cast<uint4*>(buf + lane * 32);
  const uint4 u0 = up[sw], u1 = up[sw ^ 1];
  const uint32_t uw[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
  const f2 sa2 = splat(sa);
  uint32_t dwv[8], wdu[8];
  bool rare = false;
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    dwv[q] = pack_bf16x2(mul2(mk2(__int2float_rn((int)acc[2 * q]), __int2float_rn((int)acc[2 * q + 1])), sa2));
    const int i0 = gelu_tab_index(uw[q] & 0xFFFFu), i1 = gelu_tab_index(uw[q] >> 16);
    rare |= (i0 | i1) < 0;
    wdu[q] = pack_bf16x2(mul2(unpack_bf16x2(dwv[q]), mk2(lds_f32(tab + 4u * (uint32_t)max(i0, 0)),
                                                         lds_f32(tab + 4u * (uint32_t)max(i1, 0)))));
  }
  if (__builtin_expect(rare, 0)) {  // inputs outside the table: the arithmetic itself
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const uint32_t b0 = uw[q] & 0xFFFFu, b1 = uw[q] >> 16;
      if ((gelu_tab_index(b0) | gelu_tab_index(b1)) < 0) {
        const int i0 = gelu_tab_index(b0), i1 = gelu_tab_index(b1);
        const float g0 = i0 >= 0 ? lds_f32(tab + 4u * (uint32_t)i0) : gelu_grad_slow(b0, p.act_variant);
        const float g1 = i1 >= 0 ? lds_f32(tab + 4u * (uint32_t)i1) : gelu_grad_slow(b1, p.act_variant);
        wdu[q] = pack_bf16x2(mul2(unpack_bf16x2(dwv[q]), mk2(g0, g1)));
      }
    }
  }
  up[sw] = make_uint4(wdu[0], wdu[1], wdu[2], wdu[3]);
  up[sw ^ 1] = make_uint4(wdu[4], wdu[5], wdu[6], wdu[7]);
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(tmD, buf_addr, (int32_t)fb, (int32_t)(row - lane));
    bulk_commit_group();
  }
  uint32_t a[8];
  uint32_t rw = 0u;
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    a[q] = abs_bf16x2(wdu[q]);
    if (p.colmul) {  // |v| * colmul (colmul >= 0) in fp32, as the row quantiser takes it
      float a0, a1;
      un2(mul2(unpack_bf16x2(a[q]), mk2(cm[2 * q], cm[2 * q + 1])), a0, a1);
      rmax = fmaxf(rmax, fmaxf(a0, a1));
    } else {
      rw = max_bf16x2(rw, a[q]);
    }
  }
  if (!p.colmul) rmax = fmaxf(rmax, fmaxf(__uint_as_float(rw << 16), __uint_as_float(rw & 0xFFFF0000u)));
  const uint32_t m = warp_colmax16_bits(a, lane);
  if (!(lane & 2)) atomicMax(p.col_amax + fb + colmax16_feature(lane), m);
}

template <int OUT, int BN_, int STAGES_, bool BMN>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_i8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int64_t K,
                   int tiles_m, int tiles_n, EpiParams ep) {
  extern __shared__ uint8_t smem_raw[];
  constexpr int B_BYTES_ = BN_ * BK, STAGE_BYTES_ = A_BYTES + B_BYTES_;
  constexpr int TMEM_COLS_ = ACC_STAGES * BN_ < 32 ? 32 : ACC_STAGES * BN_;
  // 1024-byte alignment for the 128B-swizzled tiles
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t pad = (1024u - (raw_addr & 1023u)) & 1023u;
  uint8_t* smem = smem_raw + pad;
  const uint32_t sbase = raw_addr + pad;
  const uint32_t sA = sbase;                    // STAGES_ x A_BYTES
  const uint32_t sB = sbase + STAGES_ * A_BYTES;  // STAGES_ x B_BYTES_
  uint8_t* ctrl = smem + STAGES_ * STAGE_BYTES_;
  const uint32_t cbase = sbase + STAGES_ * STAGE_BYTES_;
  // barrier layout (8 bytes each)
  auto full_bar = [&](int s) { return cbase + 8u * s; };
  auto empty_bar = [&](int s) { return cbase + 8u * (STAGES_ + s); };
  auto tfull_bar = [&](int a) { return cbase + 8u * (2 * STAGES_ + a); };
  auto tempty_bar = [&](int a) { return cbase + 8u * (2 * STAGES_ + ACC_STAGES + a); };
  const uint32_t drain = cbase + 8u * (2 * STAGES_ + 2 * ACC_STAGES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ctrl + 8 * (2 * STAGES_ + 2 * ACC_STAGES + 1));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(ctrl + 8 * (2 * STAGES_ + 2 * ACC_STAGES + 1) + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_kb = (int)((K + BK - 1) / BK);
  const int total_tiles = tiles_m * tiles_n;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES_; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < ACC_STAGES; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS_)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t used = 0, last_phase = 0;  // per-stage bit masks
      bool ok = true;
      for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
        int tm, tn;
        tile_coords(t, tiles_m, tiles_n, tm, tn);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!wait_bar(empty_bar(stage), phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(full_bar(stage), STAGE_BYTES_);
          tma_load_2d(sA + stage * A_BYTES, &tmA, kb * BK, tm * BM, full_bar(stage));
          if constexpr (!BMN) {
            tma_load_2d(sB + stage * B_BYTES_, &tmB, kb * BK, tn * BN_, full_bar(stage));
          } else {  // 128 k rows x 128 N bytes per box
#pragma unroll
            for (int cchunk = 0; cchunk < BN_ / 128; ++cchunk)
              tma_load_2d(sB + stage * B_BYTES_ + cchunk * (128 * BK), &tmB, tn * BN_ + cchunk * 128, kb * BK,
                          full_bar(stage));
          }
          used |= 1u << stage;
          last_phase = (last_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES_) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // make sure no TMA write into shared memory is still in flight at exit
      for (int s = 0; s < STAGES_; ++s)
        if (used & (1u << s)) drain_bar(full_bar(s), (last_phase >> s) & 1u);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      static_assert(!BMN || BN_ % 128 == 0, "MN-major B needs 128-column chunks");
      constexpr uint32_t idesc = idesc_i8(BM, BN_) | (BMN ? (1u << 16) : 0u);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
        if (!wait_bar(tempty_bar(acc), acc_phase ^ 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN_);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!wait_bar(full_bar(stage), phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = sA + stage * A_BYTES, b0 = sB + stage * B_BYTES_;
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; ++k) {
            const uint64_t bdesc = BMN ? smem_desc_mn_sw128(b0 + k * UMMA_K * 128, 128 * BK)
                                       : smem_desc_k_sw128(b0 + k * UMMA_K);
            tc_mma_i8(d_tmem, smem_desc_k_sw128(a0 + k * UMMA_K), bdesc, idesc, (kb | k) != 0);
          }
          tc_commit(empty_bar(stage));
          if (++stage == STAGES_) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(tfull_bar(acc));
        if (++acc == ACC_STAGES) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // wait until every MMA issued by this thread has finished (TMEM and smem reads)
      tc_commit(drain);
      drain_bar(drain, 0);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int lg = warp & 3;  // TMEM lane group this warp may access
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < total_tiles; t += gridDim.x) {
      int tm, tn;
      tile_coords(t, tiles_m, tiles_n, tm, tn);
      if (!__all_sync(0xffffffffu, wait_bar(tfull_bar(acc), acc_phase, abort_flag))) break;  // warp-uniform exit
      tc_fence_after();
      const int64_t row = (int64_t)tm * BM + lg * 32 + lane;
      float sa = 1.f;
      if constexpr (OUT != FF_OUT_S32) {
        if (ep.scale_a && row < ep.M) sa = __ldg(ep.scale_a + row);
      }
      const uint32_t tbase = tmem_base + ((uint32_t)(lg * 32) << 16) + (uint32_t)(acc * BN_);
      const int64_t ncol_tile = min64(BN_, ep.N - (int64_t)tn * BN_);
#pragma unroll 1
      for (int c = 0; c < BN_ / 32; ++c) {
        if ((int64_t)c * 32 >= ncol_tile) break;
        uint32_t r[32];
        tmem_ld32(tbase + c * 32, r);
        tmem_wait_ld();
        epilogue_chunk<OUT>(r, row, (int64_t)tn * BN_ + c * 32, ep, sa, lane);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty_bar(acc));
      if (++acc == ACC_STAGES) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS_)
                 : "memory");
  }
}

// ---------------------------------------------------------------------------
// 2-CTA variant: a cluster of two CTAs computes a 256 x 256 tile with
// tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 32).  Each CTA stages its own
// 128 rows of A and its own 128 rows of B (no multicast); the leader (rank 0)
// issues the MMAs, which read both CTAs' shared memory and write each CTA's
// 128 x 256 accumulator into that CTA's TMEM.  Per CTA this halves the B tile
// traffic of the 1-CTA kernel (32 KB instead of 48 KB of smem fill per k-block).
//
// Barriers: full[s] lives in the leader and completes when both CTAs' TMA loads
// of stage s landed (the leader arms it with both CTAs' bytes); empty[s] and
// tfull[a] live in both CTAs and are signalled by the leader's tcgen05.commit
// with multicast to both; tempty[a] lives in the leader and counts the 8
// epilogue warps of the pair.  All waits are time-bounded.
// ---------------------------------------------------------------------------
constexpr int C2_BM = 128;        // rows of A per CTA (256 per pair)
constexpr int C2_BN = 256;        // columns of the pair's tile (128 rows of B per CTA)
constexpr int C2_BN_CTA = 128;
constexpr int C2_STAGES = 6;
constexpr int C2_STAGES_SW = 5;  // the SwiGLU epilogue's staging buffers take one stage's space
constexpr int C2_STAGES_GELU = 4;  // the GELU epilogues also hold their value table
constexpr int C2_A_BYTES = C2_BM * BK;      // 16 KiB
constexpr int C2_B_BYTES = C2_BN_CTA * BK;  // 16 KiB
constexpr int C2_STAGE_BYTES = C2_A_BYTES + C2_B_BYTES;
constexpr int C2_SMEM_BYTES = C2_STAGES * C2_STAGE_BYTES + 1024 + 256;
// SwiGLU epilogue: per epilogue warp, two buffers (by accumulator) of the column scales and
// bias of its 64 features: gate scales, up scales, gate bias, up bias (4 x 64 floats)
constexpr int C2_SW_BUF_FLOATS = 2 * kSwigluFeat;  // per warp and buffer: its 64 features x 4 arrays
// SwiGLU: 5 stages, then 8 warps x (2 scale/bias buffers + 2 output staging buffers, 512-byte aligned)
constexpr int C2_SMEM_BYTES_SW = C2_STAGES_SW * C2_STAGE_BYTES + 1024 + 512 + 8 * 2 * C2_SW_BUF_FLOATS * 4 + 8 * 2 * 2048;
// GELU: 4 stages, the SwiGLU layout's buffers, then the table of gelu (bf16) or gelu' (fp32)
constexpr int C2_SMEM_BYTES_GELU = C2_STAGES_GELU * C2_STAGE_BYTES + 1024 + 512 + 8 * 2 * C2_SW_BUF_FLOATS * 4 +
                                   8 * 2 * 2048 + kGeluTabEntries * 4;
// bf16 output: per epilogue warp (8) two 32 x 32 bf16 staging buffers for the TMA stores (from
// byte 512 of the control area: 512-byte aligned for the 64-byte swizzle)
constexpr int C2_SMEM_BYTES_ST = C2_SMEM_BYTES + 256 + 8 * 2 * 2048;
static_assert(C2_SMEM_BYTES_ST <= 232448, "bf16-output kernel exceeds the shared memory of a CTA");
// ring epilogues: 4 stages, then the ring layout (ring_ctrl_bytes)
#ifndef FF_SWB_STAGES
#define FF_SWB_STAGES 4
#endif
constexpr int C2_STAGES_SWB = FF_SWB_STAGES;
__host__ __device__ constexpr int c2_smem_ring(int out) {
  return C2_STAGES_SWB * C2_STAGE_BYTES + 1024 + (int)ring_ctrl_bytes(out);
}
static_assert(c2_smem_ring(kOutSwigluBwd) <= 232448 && c2_smem_ring(kOutGeluBwd) <= 232448 &&
                  c2_smem_ring(kOutGeluFwd) <= 232448,
              "a wide-epilogue kernel exceeds the shared memory of a CTA");
template <int OUT>
__host__ __device__ constexpr int c2_stages() {
  return is_wide(OUT)   ? C2_STAGES_SWB
         : is_gelu(OUT) ? C2_STAGES_GELU
                              : (is_fused_act(OUT) ? C2_STAGES_SW : C2_STAGES);
}
template <int OUT>
__host__ __device__ constexpr int c2_smem_bytes() {
  return is_wide(OUT)   ? c2_smem_ring(OUT)
         : is_gelu(OUT) ? C2_SMEM_BYTES_GELU
                              : (is_fused_act(OUT) ? C2_SMEM_BYTES_SW : (OUT == FF_OUT_BF16 ? C2_SMEM_BYTES_ST : C2_SMEM_BYTES));
}
// threads of the 2-CTA kernel: TMA warp, MMA warp, then 8 epilogue warps (two per TMEM lane
// quarter, each on half of the tile's columns), so a tile's epilogue takes half as long; the
// wide epilogues run kSwbWpq warps per quarter
template <int OUT>
__host__ __device__ constexpr int c2_threads() {
  return is_wide(OUT) ? 64 + 32 * kSwbWarps : 320;
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// TMA tile load into this CTA's shared memory, completion counted on a barrier of the
// leader CTA of the pair (no multicast)
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, int32_t x, int32_t y,
                                                 uint32_t leader_bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(leader_bar)
      : "memory");
}
__device__ __forceinline__ void tc_commit_pair(uint32_t bar) {
  const uint16_t mask = 0x3;
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
                   bar),
               "h"(mask)
               : "memory");
}
__device__ __forceinline__ void tc_mma_i8_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

template <int OUT, bool BMN>
__global__ void __launch_bounds__(c2_threads<OUT>(), 1)
    gemm_i8_2cta_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmD, const __grid_constant__ CUtensorMap tmH, int64_t K,
                        int tiles_m, int tiles_n, EpiParams ep, const __grid_constant__ CUtensorMap tmB2,
                        int split) {
  constexpr int NST = c2_stages<OUT>();
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t pad = (1024u - (raw_addr & 1023u)) & 1023u;
  uint8_t* smem = smem_raw + pad;
  const uint32_t sbase = raw_addr + pad;
  const uint32_t sA = sbase;                       // NST x C2_A_BYTES
  const uint32_t sB = sbase + NST * C2_A_BYTES;  // NST x C2_B_BYTES
  uint8_t* ctrl = smem + NST * C2_STAGE_BYTES;
  const uint32_t cbase = sbase + NST * C2_STAGE_BYTES;
  auto full_bar = [&](int s) { return cbase + 8u * s; };
  auto empty_bar = [&](int s) { return cbase + 8u * (NST + s); };
  auto tfull_bar = [&](int a) { return cbase + 8u * (2 * NST + a); };
  auto tempty_bar = [&](int a) { return cbase + 8u * (2 * NST + ACC_STAGES + a); };
  const uint32_t drain = cbase + 8u * (2 * NST + 2 * ACC_STAGES);
  const uint32_t done_bar = drain + 8u;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ctrl + 8 * (2 * NST + 2 * ACC_STAGES + 2));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(ctrl + 8 * (2 * NST + 2 * ACC_STAGES + 2) + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0 = leader
  const uint32_t peer = rank ^ 1u;
  const int num_kb = (int)((K + BK - 1) / BK);
  const int total_tiles = tiles_m * tiles_n;
  const int pair = blockIdx.x >> 1, num_pairs = gridDim.x >> 1;
  // This pair's j-th tile: with `split` (plain epilogues, K-major B, a last wave at most half
  // full) the tiles of the last partial wave are cut into 256 x 128 halves, one per pair, so
  // that wave takes half the time; otherwise tile pair + j * num_pairs.  half = -1: whole tile.
  const int full_waves = split ? total_tiles / num_pairs : 0;
  const int rest = total_tiles - full_waves * num_pairs;
  auto item = [&](int j, int& tm, int& tn, int& half) -> bool {
    int t;
    half = -1;
    if (!split) {
      t = pair + j * num_pairs;
      if (t >= total_tiles) return false;
    } else if (j < full_waves) {
      t = pair + j * num_pairs;
    } else if (j == full_waves && pair < 2 * rest) {
      t = full_waves * num_pairs + (pair >> 1);
      half = pair & 1;
    } else {
      return false;
    }
    tile_coords(t, tiles_m, tiles_n, tm, tn);
    return true;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < ACC_STAGES; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 2 * (c2_threads<OUT>() / 32 - 2));  // the pair's epilogue warps
    }
    mbar_init(drain, 1);
    mbar_init(done_bar, 1);
    if constexpr (is_ring(OUT))
      for (int i = 0; i < kSwbWarps * kSwbBufs; ++i) mbar_init(cbase + ring_bar_off(OUT) + 8u * i, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  constexpr uint32_t gelu_tab_off =
      is_wide(OUT) ? ring_tab_off(OUT) : 512u + 8u * 2u * C2_SW_BUF_FLOATS * 4u + 8u * 2u * 2048u;
  if constexpr (is_gelu(OUT)) {  // the CTA's GELU table, by all threads
    for (int i = threadIdx.x; i < kGeluTabEntries; i += c2_threads<OUT>()) {
      const uint32_t b16 = gelu_tab_bits(i);
      if constexpr (OUT == kOutGeluFwd)
        reinterpret_cast<uint16_t*>(ctrl + gelu_tab_off)[i] = (uint16_t)gelu_fwd_bits_slow(b16, ep.act_variant);
      else
        reinterpret_cast<float*>(ctrl + gelu_tab_off)[i] = gelu_grad_slow(b16, ep.act_variant);
    }
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers initialised and TMEM allocated (and GELU tables filled)
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int tm, tn, half;
      for (int j = 0; ok && item(j, tm, tn, half); ++j) {
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!wait_bar(empty_bar(stage), phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t lbar = mapa_shared(full_bar(stage), 0);
          if (rank == 0)
            mbar_arrive_expect_tx(full_bar(stage), half < 0 ? 2 * C2_STAGE_BYTES : 2 * (C2_A_BYTES + C2_B_BYTES / 2));
          tma_load_2d_pair(sA + stage * C2_A_BYTES, &tmA, kb * BK, tm * (2 * C2_BM) + (int)rank * C2_BM, lbar);
          if (half >= 0) {  // this CTA's 64 rows of the half tile's 128 columns
            tma_load_2d_pair(sB + stage * C2_B_BYTES, &tmB2, kb * BK,
                             tn * C2_BN + half * (C2_BN / 2) + (int)rank * (C2_BN_CTA / 2), lbar);
          } else if constexpr (OUT == kOutSwigluFwd) {  // gate rows of the tile's features, then the up rows
            tma_load_2d_pair(sB + stage * C2_B_BYTES, &tmB, kb * BK,
                             tn * kSwigluFeat + (rank ? (int)ep.F : 0), lbar);
          } else if constexpr (!BMN) {
            tma_load_2d_pair(sB + stage * C2_B_BYTES, &tmB, kb * BK, tn * C2_BN + (int)rank * C2_BN_CTA, lbar);
          } else {  // this CTA's 128 columns of B: 128 k rows x 128 N bytes
            tma_load_2d_pair(sB + stage * C2_B_BYTES, &tmB, tn * C2_BN + (int)rank * C2_BN_CTA, kb * BK, lbar);
          }
          if (++stage == NST) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader only)
    if (rank == 0 && lane == 0) {
      constexpr uint32_t idesc = idesc_i8(2 * C2_BM, C2_BN) | (BMN ? (1u << 16) : 0u);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      constexpr uint32_t idesc_half = idesc_i8(2 * C2_BM, C2_BN / 2);
      int tm_, tn_, half;
      for (int j = 0; ok && item(j, tm_, tn_, half); ++j) {
        if (!wait_bar(tempty_bar(acc), acc_phase ^ 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * C2_BN);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!wait_bar(full_bar(stage), phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = sA + stage * C2_A_BYTES, b0 = sB + stage * C2_B_BYTES;
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; ++k) {
            const uint64_t bdesc = BMN ? smem_desc_mn_sw128(b0 + k * UMMA_K * 128, 128 * BK)
                                       : smem_desc_k_sw128(b0 + k * UMMA_K);
            tc_mma_i8_pair(d_tmem, smem_desc_k_sw128(a0 + k * UMMA_K), bdesc, half < 0 ? idesc : idesc_half,
                           (kb | k) != 0);
          }
          tc_commit_pair(empty_bar(stage));  // frees the stage in both CTAs
          if (++stage == NST) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit_pair(tfull_bar(acc));  // accumulator ready in both CTAs
        if (++acc == ACC_STAGES) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      tc_commit(drain);  // every MMA of this thread has finished
      drain_bar(drain, 0);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int lg = warp & 3;           // TMEM lane quarter
    const int eh = (warp - 2) >> 2;    // SwiGLU: which half of the tile's features (0 or 1)
    int acc = 0;
    uint32_t acc_phase = 0;
    // SwiGLU: this warp's two staging buffers of its features' column scales and bias (the
    // backward epilogue: one buffer of its column multipliers)
    constexpr int sw_bufs = is_wide(OUT) ? 1 : 2;
    float* sw_buf = is_wide(OUT) ? reinterpret_cast<float*>(ctrl + kSwbCmOff + (warp - 2) * ring_cm_bytes(OUT))
                                 : reinterpret_cast<float*>(ctrl + 256) + (warp - 2) * sw_bufs * C2_SW_BUF_FLOATS;
    // this warp's two TMA-store staging buffers (32 rows x 64 B each, 512-byte aligned for the
    // 64-byte swizzle); with the activation epilogues they follow the 8 warps' scale/bias buffers
    constexpr uint32_t st_off = 512u + (is_fused_act(OUT) ? 8u * 2u * C2_SW_BUF_FLOATS * 4u : 0u);
    uint8_t* st_stage = ctrl + st_off + (warp - 2) * 2 * 2048;
    const uint32_t st_stage_addr = cbase + st_off + (uint32_t)(warp - 2) * 2 * 2048;
    uint32_t st_count = 0;
    int tm, tn, half;
    // ring epilogues: this warp's ring of input chunks (kSwbChunk).  The warp's chunks (those of
    // its chunk indices that lie below F) in schedule order; lane 0 keeps the cursor of the next
    // chunk to load (item sj, chunk sc at tile sm, sn) and the count of chunks loaded.
    constexpr int kRingBuf = ring_buf_bytes(OUT);
    constexpr int kRingBufs = ring_bufs(OUT);
    [[maybe_unused]] const uint32_t swb_ring = cbase + ring_off(OUT) + (uint32_t)(warp - 2) * kRingBufs * kRingBuf;
    [[maybe_unused]] uint8_t* swb_ring_p = ctrl + ring_off(OUT) + (warp - 2) * kRingBufs * kRingBuf;
    [[maybe_unused]] const uint32_t swb_bar = cbase + ring_bar_off(OUT) + (uint32_t)(warp - 2) * kRingBufs * 8;
    // chunks of tile column tn below F (16, or 8 for a last tile of 128 features: F % 128 == 0)
    auto swb_chunks = [&](int tn_) { return (int)min64(C2_BN / kSwbChunk, (ep.F - (int64_t)tn_ * C2_BN) / kSwbChunk); };
    int sj = 0, sc = 0, sm = 0, sn = 0, swb_loaded = 0, swb_used = 0;
    bool s_ok = false;
    auto swb_seek = [&](int from) {  // the first item >= from with a chunk of this warp
      int h_;
      for (sj = from; item(sj, sm, sn, h_); ++sj)
        if (swb_chunks(sn) > eh) {
          sc = eh;
          s_ok = true;
          return;
        }
      s_ok = false;
    };
    auto swb_load = [&]() {  // lane 0: TMA loads of the cursor's chunk into its ring buffer
      const int b = swb_loaded % kSwbBufs;
      const int32_t x = (int32_t)((int64_t)sn * C2_BN + sc * kSwbChunk);
      const int32_t y = (int32_t)((int64_t)sm * (2 * C2_BM) + (int64_t)rank * C2_BM + lg * 32);
      const uint32_t bar = swb_bar + 8u * (uint32_t)b, dst = swb_ring + (uint32_t)(b * kRingBuf);
      mbar_arrive_expect_tx(bar, kRingBuf);
      tma_load_2d(dst, &tmH, x, y, bar);  // SwiGLU: g; GELU: u
      if constexpr (OUT == kOutSwigluBwd) tma_load_2d(dst + kSwbBoxBytes, &tmH, (int32_t)ep.F + x, y, bar);  // u
      ++swb_loaded;
      sc += kSwbWpq;
      if (sc >= swb_chunks(sn)) swb_seek(sj + 1);
    };
    if constexpr (is_ring(OUT)) {
      if (lane == 0) {
        swb_seek(0);
        while (s_ok && swb_loaded < kSwbBufs) swb_load();
      }
    }
    bool swb_abort = false;
    for (int j = 0; item(j, tm, tn, half); ++j) {
      float4 st_s, st_b;  // loaded before the accumulator wait, stored after it
      [[maybe_unused]] float4 st_s2, st_b2;  // ring epilogues: the multipliers of features 128..255
      if constexpr (OUT == kOutSwigluBwd) {
        // the tile's 256 features: lane l holds gate multipliers 4l..4l+3 and 128+4l..128+4l+3, up likewise
        const int64_t col = (int64_t)tn * C2_BN + lane * 4;
        const bool in = ep.colmul && col < ep.F, in2 = ep.colmul && col + 128 < ep.F;
        const float4 one4 = make_float4(1.f, 1.f, 1.f, 1.f);
        st_s = in ? __ldg(reinterpret_cast<const float4*>(ep.colmul + col)) : one4;
        st_b = in ? __ldg(reinterpret_cast<const float4*>(ep.colmul + ep.F + col)) : one4;
        st_s2 = in2 ? __ldg(reinterpret_cast<const float4*>(ep.colmul + col + 128)) : one4;
        st_b2 = in2 ? __ldg(reinterpret_cast<const float4*>(ep.colmul + ep.F + col + 128)) : one4;
      }
      if constexpr (OUT == kOutGeluBwd) {
        // the tile's 256 features: lane l holds the multipliers of features 4l..4l+3 and 128+4l..128+4l+3
        const int64_t col = (int64_t)tn * C2_BN + lane * 4;
        const bool in = ep.colmul && col < ep.F, in2 = ep.colmul && col + 128 < ep.F;
        const float4 one4 = make_float4(1.f, 1.f, 1.f, 1.f);
        st_s = in ? __ldg(reinterpret_cast<const float4*>(ep.colmul + col)) : one4;
        st_s2 = in2 ? __ldg(reinterpret_cast<const float4*>(ep.colmul + col + 128)) : one4;
      }
      if constexpr (OUT == kOutGeluFwd) {
        // the tile's 256 features: lane l holds the column scales and biases of features 4l..4l+3 and
        // 128+4l..128+4l+3
        const int64_t col = (int64_t)tn * C2_BN + lane * 4;
        const bool in = col < ep.F, in2 = col + 128 < ep.F;
        // missing scales are 1 and a missing bias -0: x * 1 and x + (-0) give x exactly, signed zeros included
        const float4 one4 = make_float4(1.f, 1.f, 1.f, 1.f), nzero4 = make_float4(-0.f, -0.f, -0.f, -0.f);
        st_s = in && ep.scale_b ? __ldg(reinterpret_cast<const float4*>(ep.scale_b + col)) : one4;
        st_s2 = in2 && ep.scale_b ? __ldg(reinterpret_cast<const float4*>(ep.scale_b + col + 128)) : one4;
        st_b = in && ep.bias ? __ldg(reinterpret_cast<const float4*>(ep.bias + col)) : nzero4;
        st_b2 = in2 && ep.bias ? __ldg(reinterpret_cast<const float4*>(ep.bias + col + 128)) : nzero4;
      }
      if constexpr (OUT == kOutSwigluFwd) {
        // lanes 0-15: the 64 gate features of this warp, lanes 16-31: the same 64 up features
        const int64_t col = (int64_t)(lane >> 4) * ep.F + (int64_t)tn * kSwigluFeat + eh * 64 + (lane & 15) * 4;
        st_s = ep.scale_b ? __ldg(reinterpret_cast<const float4*>(ep.scale_b + col)) : make_float4(1.f, 1.f, 1.f, 1.f);
        st_b = ep.bias ? __ldg(reinterpret_cast<const float4*>(ep.bias + col)) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      if (!__all_sync(0xffffffffu, wait_bar(tfull_bar(acc), acc_phase, abort_flag))) break;  // warp-uniform exit
      tc_fence_after();
      if constexpr (is_fused_act(OUT)) {
        float* buf = sw_buf + (sw_bufs == 2 ? acc : 0) * C2_SW_BUF_FLOATS;
        if constexpr (OUT == kOutSwigluBwd || OUT == kOutGeluFwd) {  // [gate 256 | up 256], [scale 256 | bias 256]
          reinterpret_cast<float4*>(buf)[lane] = st_s;
          reinterpret_cast<float4*>(buf + 128)[lane] = st_s2;
          reinterpret_cast<float4*>(buf + 256)[lane] = st_b;
          reinterpret_cast<float4*>(buf + 384)[lane] = st_b2;
        } else if constexpr (OUT == kOutGeluBwd) {  // [256]
          reinterpret_cast<float4*>(buf)[lane] = st_s;
          reinterpret_cast<float4*>(buf + 128)[lane] = st_s2;
        } else {
          reinterpret_cast<float4*>(buf)[lane] = st_s;       // [gate 64 | up 64]
          reinterpret_cast<float4*>(buf + 128)[lane] = st_b;  // [gate bias 64 | up bias 64]
        }
        __syncwarp();
      }
      const int64_t row = (int64_t)tm * (2 * C2_BM) + (int64_t)rank * C2_BM + lg * 32 + lane;
      float sa = 1.f;
      if constexpr (OUT != FF_OUT_S32) {
        if (ep.scale_a && row < ep.M) sa = __ldg(ep.scale_a + row);
      }
      const uint32_t tbase = tmem_base + ((uint32_t)(lg * 32) << 16) + (uint32_t)(acc * C2_BN);
      if constexpr (OUT == kOutSwigluFwd) {
        uint32_t rmax = 0u;
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {  // this warp's 64 features: two chunks of 32
          const int fc = eh * 64 + c * 32;
          uint32_t rg[32], ru[32];
          tmem_ld32(tbase + fc, rg);
          tmem_ld32(tbase + kSwigluFeat + fc, ru);
          tmem_wait_ld();
          swiglu_fwd_chunk(rg, ru, row, (int64_t)tn * kSwigluFeat + fc, ep, sa, lane,
                           sw_buf + acc * C2_SW_BUF_FLOATS + c * 32, rmax, &tmD, &tmH, st_stage, st_stage_addr,
                           st_count);
        }
        if (row < ep.M)
          atomicMax(ep.row_amax + row, __float_as_uint(fmaxf(__uint_as_float(rmax << 16),
                                                               __uint_as_float(rmax & 0xFFFF0000u))));
      } else if constexpr (OUT == kOutGeluFwd) {
        const int nchunks = swb_chunks(tn);
        if (nchunks > eh) {
          uint32_t rmax = 0u;
          const float* cmb = sw_buf;  // [scale 256 | bias 256] of the tile's features
#pragma unroll 1
          for (int c = eh; c < nchunks; c += kSwbWpq, ++swb_used) {
            const int b = swb_used & 1;
            if (swb_used >= 2) {  // this buffer's stores (two chunks ago) must have read it
              if (lane == 0) bulk_wait_read_1();
              __syncwarp();
            }
            uint32_t r[16];
            tmem_ld16(tbase + c * kSwbChunk, r);
            tmem_wait_ld();
            gelu_fwd_chunk16(r, swb_ring_p + b * kRingBuf, swb_ring + (uint32_t)(b * kRingBuf), row,
                             (int64_t)tn * C2_BN + c * kSwbChunk, ep, sa, lane, cmb + c * kSwbChunk,
                             cmb + 256 + c * kSwbChunk, cbase + gelu_tab_off, rmax, &tmD, &tmH);
          }
          if (row < ep.M)
            atomicMax(ep.row_amax + row, __float_as_uint(fmaxf(__uint_as_float(rmax << 16),
                                                                 __uint_as_float(rmax & 0xFFFF0000u))));
        }
      } else if constexpr (is_ring(OUT)) {
        const int nchunks = swb_chunks(tn);
        if (nchunks > eh) {
          float rmax = 0.f;
          const float* cmb = sw_buf;  // the multipliers of the tile's features ([gate 256 | up 256], or [256])
#pragma unroll 1
          for (int c = eh; c < nchunks; c += kSwbWpq, ++swb_used) {
            const int b = swb_used % kSwbBufs;
            // warp-uniform: lanes that saw the phase complete leave with those that saw the abort
            if (!__all_sync(0xffffffffu, wait_bar(swb_bar + 8u * (uint32_t)b, (uint32_t)(swb_used / kSwbBufs) & 1u,
                                                  abort_flag))) {
              swb_abort = true;
              break;
            }
            uint32_t r[16];
            tmem_ld16(tbase + c * kSwbChunk, r);
            tmem_wait_ld();
            const int64_t fb = (int64_t)tn * C2_BN + c * kSwbChunk;
            if constexpr (OUT == kOutSwigluBwd)
              swiglu_bwd_chunk16(r, swb_ring_p + b * kRingBuf, swb_ring + (uint32_t)(b * kRingBuf), row, fb, ep, sa,
                                 lane, cmb + c * kSwbChunk, cmb + 256 + c * kSwbChunk, rmax, &tmD);
            else
              gelu_bwd_chunk16(r, swb_ring_p + b * kRingBuf, swb_ring + (uint32_t)(b * kRingBuf), row, fb, ep, sa, lane,
                               cmb + c * kSwbChunk, cbase + gelu_tab_off, rmax, &tmD);
            // the previous chunk's buffer (its stores were issued one chunk ago) takes the chunk
            // kSwbBufs - 1 ahead of the next
            if (lane == 0 && swb_used >= 1 && s_ok) {
              bulk_wait_read_1();
              swb_load();
            }
            __syncwarp();
          }
          if (row < ep.M) atomicMax(ep.row_amax + row, __float_as_uint(rmax));
        }
        if (swb_abort) break;
      } else {
        const int64_t col0 = (int64_t)tn * C2_BN + (half < 0 ? 0 : half * (C2_BN / 2));
        const int64_t ncol_tile = min64(half < 0 ? C2_BN : C2_BN / 2, ep.N - col0);
        // this warp's half of the tile's 32-column chunks
        const int nchunk = (half < 0 ? C2_BN : C2_BN / 2) / 64;
#pragma unroll 1
        for (int c = eh * nchunk; c < (eh + 1) * nchunk; ++c) {
          if ((int64_t)c * 32 >= ncol_tile) break;
          uint32_t r[32];
          tmem_ld32(tbase + c * 32, r);
          tmem_wait_ld();
          if constexpr (OUT == FF_OUT_BF16) {
            if (ep.tma_store) {
              epilogue_chunk_tma(r, col0 + c * 32, row - lane, ep, &tmD, sa, lane, st_stage, st_stage_addr, st_count);
              continue;
            }
          }
          epilogue_chunk<OUT>(r, row, col0 + c * 32, ep, sa, lane);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(mapa_shared(tempty_bar(acc), 0));
      if (++acc == ACC_STAGES) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if ((st_count || is_wide(OUT)) && lane == 0) bulk_wait_all();  // TMA stores complete before the CTA exits
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (*abort_flag) spin_ns(20000);  // let any TMA load still in flight land before the CTA exits
  // neither CTA frees TMEM before the other is done with the pair's allocation
  if (threadIdx.x == 32) {
    mbar_arrive_remote(mapa_shared(done_bar, peer));
    drain_bar(done_bar, 0);
  }
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                 : "memory");
  }
}

}  // namespace gemm
}  // namespace ff

#include "ff_gemm_skinny.cuh"

namespace ff {
namespace gemm {

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
inline int make_map(CUtensorMap* m, const int8_t* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return set_error(FF_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(FF_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return FF_OK;
}

// bf16 output [rows, cols] (leading dim ld) for TMA tile stores of 32 x 32 boxes
inline int make_map_out_bf16(CUtensorMap* m, void* ptr, int64_t rows, int64_t cols, int64_t ld, bool swz64 = false) {
  return make_map_bf16(m, ptr, rows, cols, ld, 32, 32, swz64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_NONE);
}

inline int num_sms_current() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!cache[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

template <int OUT, int BN_, int STAGES_, bool BMN>
inline int launch(const CUtensorMap& ma, const CUtensorMap& mb, int64_t K, int tiles_m, int tiles_n,
                  const EpiParams& ep, int grid, cudaStream_t st) {
  constexpr int smem = STAGES_ * (A_BYTES + BN_ * BK) + 1024 + 256;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    FF_CUDA_TRY(cudaFuncSetAttribute(gemm_i8_kernel<OUT, BN_, STAGES_, BMN>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                "ff_gemm_i8 smem attribute");
    attr_set[dev] = true;
  }
  gemm_i8_kernel<OUT, BN_, STAGES_, BMN><<<grid, NUM_THREADS, smem, st>>>(ma, mb, K, tiles_m, tiles_n, ep);
  return check_launch("ff_gemm_i8");
}

// narrow tiles (128 x 64, 8 stages) for problems that 128 x 256 tiles cannot spread over the SMs
constexpr int NARROW_BN = 64;
constexpr int NARROW_STAGES = 8;

template <int OUT, bool BMN>
inline int launch_2cta(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& md, const CUtensorMap& mh,
                       int64_t K, int tiles_m, int tiles_n, const EpiParams& ep, int max_pairs, cudaStream_t st,
                       const CUtensorMap* mb2 = nullptr) {
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    FF_CUDA_TRY(cudaFuncSetAttribute(gemm_i8_2cta_kernel<OUT, BMN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     c2_smem_bytes<OUT>()),
                "ff_gemm_i8 2-CTA smem attribute");
    attr_set[dev] = true;
  }
  const int pairs = min(tiles_m * tiles_n, max_pairs);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * pairs));
  cfg.blockDim = dim3(c2_threads<OUT>());
  cfg.dynamicSmemBytes = c2_smem_bytes<OUT>();
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // the last wave of tiles cut into halves when it is at most half full (plain epilogues, K-major B)
  const int total = tiles_m * tiles_n, rest = total % pairs;
  const int split = (mb2 != nullptr && !BMN && OUT <= FF_OUT_BF16_ACCUM && total > pairs && rest > 0 &&
                     2 * rest <= pairs) ? 1 : 0;
  FF_CUDA_TRY(cudaLaunchKernelEx(&cfg, gemm_i8_2cta_kernel<OUT, BMN>, ma, mb, md, mh, K, tiles_m, tiles_n, ep,
                                 mb2 ? *mb2 : mb, split),
              "ff_gemm_i8 2-CTA launch");
  return check_launch("ff_gemm_i8 (2-CTA)");
}

// clusters of two 2-CTA GEMM CTAs that fit on the device at once (cached per device)
inline int max_pairs_current() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  if (!cache[dev]) {
    cudaFuncSetAttribute(gemm_i8_2cta_kernel<FF_OUT_BF16, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         c2_smem_bytes<FF_OUT_BF16>());
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2);
    cfg.blockDim = dim3(c2_threads<FF_OUT_BF16>());
    cfg.dynamicSmemBytes = c2_smem_bytes<FF_OUT_BF16>();
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_i8_2cta_kernel<FF_OUT_BF16, false>, &cfg) != cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
    cache[dev] = n > 0 ? n : -1;
  }
  return cache[dev] > 0 ? cache[dev] : 0;
}

// One GEMM, any layout of B: BMN == false -> B is N x K (ldb), BMN == true -> B is K x N (ldb).
// Skinny problems (M <= 128, K-major B) given a workspace of at least skinny_ws_bytes(M, N) bytes
// take the stream-K kernel of ff_gemm_skinny.cuh.
template <bool BMN>
inline int gemm_dispatch(const char* name, const int8_t* A, int64_t lda, const int8_t* B, int64_t ldb,
                         const float* scale_a, const float* scale_b, const float* bias, void* D, int64_t ldd,
                         int out_kind, int64_t M, int64_t N, int64_t K, void* stream, void* ws = nullptr,
                         int64_t ws_bytes = 0) {
  FF_REQUIRE(M >= 0 && N >= 0 && K >= 1, FF_ERR_INVALID_ARG, "%s: M=%lld N=%lld K=%lld", name, (long long)M,
             (long long)N, (long long)K);
  FF_REQUIRE(out_kind >= FF_OUT_S32 && out_kind <= FF_OUT_BF16_ACCUM, FF_ERR_INVALID_ARG, "%s: bad out_kind %d", name,
             out_kind);
  if (M == 0 || N == 0) return FF_OK;
  FF_REQUIRE(A && B && D, FF_ERR_INVALID_ARG, "%s: null pointer", name);
  FF_REQUIRE(lda >= K && ldb >= (BMN ? N : K) && ldd >= N, FF_ERR_INVALID_ARG, "%s: bad leading dims", name);
  FF_REQUIRE(aligned(A, 16) && aligned(B, 16) && lda % 16 == 0 && ldb % 16 == 0, FF_ERR_UNSUPPORTED,
             "%s: A/B need 16-byte alignment and lda/ldb multiples of 16 (lda=%lld ldb=%lld)", name,
             (long long)lda, (long long)ldb);
  FF_REQUIRE(M <= (int64_t)1 << 31 && N <= (int64_t)1 << 31 && K <= (int64_t)1 << 31, FF_ERR_UNSUPPORTED,
             "%s: dimension too large", name);
  const int64_t tm64 = (M + BM - 1) / BM, tn64 = (N + BN - 1) / BN;
  FF_REQUIRE(tm64 * tn64 < ((int64_t)1 << 31), FF_ERR_UNSUPPORTED, "%s: too many tiles", name);
  cudaStream_t st = as_stream(stream);
  CUtensorMap ma, mb;
  int rc = make_map(&ma, A, M, K, lda, BM);
  if (rc) return rc;
  const int es = (out_kind == FF_OUT_BF16 || out_kind == FF_OUT_BF16_ACCUM) ? 2 : 4;
  EpiParams ep{};
  ep.scale_a = scale_a;
  ep.scale_b = scale_b;
  ep.bias = bias;
  ep.D = D;
  ep.ldd = ldd;
  ep.M = M;
  ep.N = N;
  ep.vec = aligned(D, 16) && ((ldd * es) % 16 == 0);
  if constexpr (!BMN) {
    if (ws && M <= 128) {
      const int mp = sk_mp(M);
      const int64_t tiles = (N + SK_BN - 1) / SK_BN;
      FF_REQUIRE(ws_bytes >= sk_ws_bytes(tiles, mp) && aligned(ws, 16), FF_ERR_INVALID_ARG,
                 "%s: workspace of %lld bytes (16-byte aligned) needed, got %lld", name,
                 (long long)sk_ws_bytes(tiles, mp), (long long)ws_bytes);
      rc = make_map(&mb, B, N, K, ldb, SK_BN);
      if (rc) return rc;
      CUtensorMap mas;
      rc = make_map(&mas, A, M, K, lda, mp);
      if (rc) return rc;
      const int64_t total = tiles * ((K + BK - 1) / BK);
      const int grid = (int)min64((int64_t)num_sms_current(), max64(1, total / 2));
      int32_t* part = static_cast<int32_t*>(ws);
      uint32_t* cnt = reinterpret_cast<uint32_t*>(part + tiles * mp * SK_BN);
      switch (out_kind) {
        case FF_OUT_S32: return launch_skinny_mp<FF_OUT_S32>(mp, mas, mb, K, (int)tiles, ep, grid, part, cnt, st);
        case FF_OUT_F32: return launch_skinny_mp<FF_OUT_F32>(mp, mas, mb, K, (int)tiles, ep, grid, part, cnt, st);
        case FF_OUT_BF16: return launch_skinny_mp<FF_OUT_BF16>(mp, mas, mb, K, (int)tiles, ep, grid, part, cnt, st);
        default: return launch_skinny_mp<FF_OUT_BF16_ACCUM>(mp, mas, mb, K, (int)tiles, ep, grid, part, cnt, st);
      }
    }
  }
  // Tile configuration by a small cost model: waves x work per SM per tile / relative
  // efficiency, for 256 x 256 tiles on CTA pairs (cta_group::2), 128 x 256 tiles and
  // 128 x 64 tiles (the narrow tiles spread small and skinny problems over the SMs; not
  // offered for an MN-major B, which is staged in 128-column chunks).
  const int nsm = num_sms_current();
  const int max_pairs = (M >= 256 && N >= 256) ? max_pairs_current() : 0;
  const int64_t pair_tiles = ((M + 255) / 256) * ((N + 255) / 256);
  const int64_t wide_tiles = tm64 * tn64;
  const int64_t narrow_tiles = tm64 * ((N + 63) / 64);
  auto waves = [](int64_t tiles, int64_t slots) { return (double)((tiles + slots - 1) / slots); };
  // pair tiles: a last wave at most half full is cut into half-width tiles (plain epilogues, K-major
  // B), so it costs half a wave
  auto pair_waves = [&]() {
    const int64_t full = pair_tiles / max_pairs, rest = pair_tiles % max_pairs;
    if (!BMN && full > 0 && rest > 0 && 2 * rest <= max_pairs) return (double)full + 0.5;
    return waves(pair_tiles, max_pairs);
  };
  const double cost_pair = max_pairs > 0 ? pair_waves() * 4.0 : 1e300;
  const double cost_wide = waves(wide_tiles, nsm) * 4.0 / 0.9;
  const double cost_narrow = BMN ? 1e300 : waves(narrow_tiles, nsm) * 1.0 / 0.6;
  // B maps: K-major boxes are (128 K bytes) x (rows of N); MN-major boxes are (128 N bytes) x (128 K rows)
  auto map_b = [&](int n_rows_per_box) {
    return BMN ? make_map(&mb, B, K, N, ldb, BK) : make_map(&mb, B, N, K, ldb, n_rows_per_box);
  };
  if (cost_pair <= cost_wide && cost_pair <= cost_narrow) {
    rc = map_b(C2_BN_CTA);
    if (rc) return rc;
    const int t2m = (int)((M + 2 * C2_BM - 1) / (2 * C2_BM)), t2n = (int)((N + C2_BN - 1) / C2_BN);
    CUtensorMap md;
    memset(&md, 0, sizeof(md));
    if (out_kind == FF_OUT_BF16 && ep.vec) {  // 16-byte aligned output rows: TMA tile stores
      rc = make_map_out_bf16(&md, D, M, N, ldd, true);
      if (rc) return rc;
      ep.tma_store = 1;
    }
    CUtensorMap mb2;  // 64-row boxes of B for the half-width tiles of a short last wave
    const CUtensorMap* pmb2 = nullptr;
    if constexpr (!BMN) {
      rc = make_map(&mb2, B, N, K, ldb, C2_BN_CTA / 2);
      if (rc) return rc;
      pmb2 = &mb2;
    }
    switch (out_kind) {
      case FF_OUT_S32: return launch_2cta<FF_OUT_S32, BMN>(ma, mb, md, md, K, t2m, t2n, ep, max_pairs, st, pmb2);
      case FF_OUT_F32: return launch_2cta<FF_OUT_F32, BMN>(ma, mb, md, md, K, t2m, t2n, ep, max_pairs, st, pmb2);
      case FF_OUT_BF16: return launch_2cta<FF_OUT_BF16, BMN>(ma, mb, md, md, K, t2m, t2n, ep, max_pairs, st, pmb2);
      default:
        return launch_2cta<FF_OUT_BF16_ACCUM, BMN>(ma, mb, md, md, K, t2m, t2n, ep, max_pairs, st, pmb2);
    }
  }
  if (cost_wide <= cost_narrow) {  // 128 x 256 tiles, one CTA each
    rc = map_b(BN);
    if (rc) return rc;
    const int tiles_m = (int)tm64, tiles_n = (int)tn64;
    const int grid = min(tiles_m * tiles_n, nsm);
    switch (out_kind) {
      case FF_OUT_S32: return launch<FF_OUT_S32, BN, STAGES, BMN>(ma, mb, K, tiles_m, tiles_n, ep, grid, st);
      case FF_OUT_F32: return launch<FF_OUT_F32, BN, STAGES, BMN>(ma, mb, K, tiles_m, tiles_n, ep, grid, st);
      case FF_OUT_BF16: return launch<FF_OUT_BF16, BN, STAGES, BMN>(ma, mb, K, tiles_m, tiles_n, ep, grid, st);
      default: return launch<FF_OUT_BF16_ACCUM, BN, STAGES, BMN>(ma, mb, K, tiles_m, tiles_n, ep, grid, st);
    }
  }
  if constexpr (!BMN) {
    // small or skinny problems: 128 x 64 tiles (skinny M streams B at HBM speed over many SMs)
    rc = map_b(NARROW_BN);
    if (rc) return rc;
    const int tiles_m = (int)tm64, tiles_n = (int)((N + NARROW_BN - 1) / NARROW_BN);
    FF_REQUIRE((int64_t)tiles_m * tiles_n < ((int64_t)1 << 31), FF_ERR_UNSUPPORTED, "%s: too many tiles", name);
    const int grid = min(tiles_m * tiles_n, nsm);
    switch (out_kind) {
      case FF_OUT_S32:
        return launch<FF_OUT_S32, NARROW_BN, NARROW_STAGES, false>(ma, mb, K, tiles_m, tiles_n, ep, grid, st);
      case FF_OUT_F32:
        return launch<FF_OUT_F32, NARROW_BN, NARROW_STAGES, false>(ma, mb, K, tiles_m, tiles_n, ep, grid, st);
      case FF_OUT_BF16:
        return launch<FF_OUT_BF16, NARROW_BN, NARROW_STAGES, false>(ma, mb, K, tiles_m, tiles_n, ep, grid, st);
      default:
        return launch<FF_OUT_BF16_ACCUM, NARROW_BN, NARROW_STAGES, false>(ma, mb, K, tiles_m, tiles_n, ep, grid,
                                                                          st);
    }
  }
  return set_error(FF_ERR_UNSUPPORTED, "%s: no tile configuration", name);
}

}  // namespace gemm
}  // namespace ff

extern "C" int ff_gemm_i8(const int8_t* A, int64_t lda, const int8_t* B, int64_t ldb, const float* scale_a,
                          const float* scale_b, const float* bias, void* D, int64_t ldd, int out_kind, int64_t M,
                          int64_t N, int64_t K, void* stream) {
  return ff::gemm::gemm_dispatch<false>("ff_gemm_i8", A, lda, B, ldb, scale_a, scale_b, bias, D, ldd, out_kind, M, N,
                                        K, stream);
}

extern "C" int64_t ff_gemm_i8_ws_bytes(int64_t M, int64_t N, int64_t K) {
  if (M < 1 || M > 128 || N < 1 || K < 1) return 0;
  return ff::gemm::sk_ws_bytes((N + ff::gemm::SK_BN - 1) / ff::gemm::SK_BN, ff::gemm::sk_mp(M));
}

extern "C" int ff_gemm_i8_ws(const int8_t* A, int64_t lda, const int8_t* B, int64_t ldb, const float* scale_a,
                             const float* scale_b, const float* bias, void* D, int64_t ldd, int out_kind, int64_t M,
                             int64_t N, int64_t K, void* ws, int64_t ws_bytes, void* stream) {
  return ff::gemm::gemm_dispatch<false>("ff_gemm_i8_ws", A, lda, B, ldb, scale_a, scale_b, bias, D, ldd, out_kind, M,
                                        N, K, stream, ws, ws_bytes);
}

extern "C" int ff_swiglu_gemm_i8(const int8_t* A, int64_t lda, const int8_t* B, int64_t ldb, const float* scale_a,
                                 const float* scale_b, const float* bias, uint16_t* gu, int64_t ldgu, uint16_t* h,
                                 int64_t ldh, int64_t M, int64_t F, int64_t K, float eps, int8_t* q_rows, int64_t ldq,
                                 float* s_rows, int8_t* q_cols_t, int64_t ldqt, float* s_cols, float* absmax_ws,
                                 void* stream) {
  using namespace ff;
  using namespace ff::gemm;
  const char* name = "ff_swiglu_gemm_i8";
  FF_REQUIRE(M >= 0 && F >= 1 && K >= 1, FF_ERR_INVALID_ARG, "%s: M=%lld F=%lld K=%lld", name, (long long)M,
             (long long)F, (long long)K);
  FF_REQUIRE(F % kSwigluFeat == 0, FF_ERR_UNSUPPORTED, "%s: F=%lld must be a multiple of %d", name, (long long)F,
             kSwigluFeat);
  FF_REQUIRE(q_rows || q_cols_t, FF_ERR_INVALID_ARG, "%s: nothing to do", name);
  if (M == 0) return FF_OK;
  FF_REQUIRE(A && B && gu && h, FF_ERR_INVALID_ARG, "%s: null pointer", name);
  FF_REQUIRE(lda >= K && ldb >= K && ldgu >= 2 * F && ldh >= F, FF_ERR_INVALID_ARG, "%s: bad leading dims", name);
  FF_REQUIRE(aligned(A, 16) && aligned(B, 16) && lda % 16 == 0 && ldb % 16 == 0, FF_ERR_UNSUPPORTED,
             "%s: A/B need 16-byte alignment and lda/ldb multiples of 16", name);
  FF_REQUIRE(aligned(gu, 16) && aligned(h, 16) && ldgu % 8 == 0 && ldh % 8 == 0, FF_ERR_UNSUPPORTED,
             "%s: gu/h need 16-byte alignment and leading dims multiples of 8", name);
  FF_REQUIRE((!scale_b || aligned(scale_b, 16)) && (!bias || aligned(bias, 16)), FF_ERR_UNSUPPORTED,
             "%s: scale_b/bias need 16-byte alignment", name);
  FF_REQUIRE(M <= (int64_t)1 << 31 && 2 * F <= (int64_t)1 << 31 && K <= (int64_t)1 << 31, FF_ERR_UNSUPPORTED,
             "%s: dimension too large", name);
  int rc = check_dual_outputs(name, M, F, q_rows, ldq, s_rows, q_cols_t, ldqt, s_cols, absmax_ws);
  if (rc != FF_OK) return rc;
  const int max_pairs = max_pairs_current();
  FF_REQUIRE(max_pairs > 0, FF_ERR_UNSUPPORTED, "%s: the 2-CTA GEMM cannot be resident on this device", name);
  cudaStream_t st = as_stream(stream);
  FF_CUDA_TRY(cudaMemsetAsync(absmax_ws, 0, sizeof(float) * (size_t)(M + F), st), name);
  CUtensorMap ma, mb;
  rc = make_map(&ma, A, M, K, lda, BM);
  if (rc) return rc;
  rc = make_map(&mb, B, 2 * F, K, ldb, C2_BN_CTA);
  if (rc) return rc;
  EpiParams ep{};
  ep.scale_a = scale_a;
  ep.scale_b = scale_b;
  ep.bias = bias;
  ep.D = gu;
  ep.ldd = ldgu;
  ep.M = M;
  ep.N = 2 * F;
  ep.vec = 1;
  ep.h = reinterpret_cast<__nv_bfloat16*>(h);
  ep.ldh = ldh;
  ep.F = F;
  ep.row_amax = reinterpret_cast<uint32_t*>(absmax_ws);
  ep.col_amax = ep.row_amax + M;
  const int t2m = (int)((M + 2 * C2_BM - 1) / (2 * C2_BM)), t2n = (int)(F / kSwigluFeat);
  CUtensorMap md, mh;  // gu and h, written by TMA tile stores
  rc = make_map_out_bf16(&md, gu, M, 2 * F, ldgu, true);
  if (rc) return rc;
  rc = make_map_out_bf16(&mh, h, M, F, ldh, true);
  if (rc) return rc;
  rc = launch_2cta<kOutSwigluFwd, false>(ma, mb, md, mh, K, t2m, t2n, ep, max_pairs, st);
  if (rc != FF_OK) return rc;
  return launch_pass_b<FF_DTYPE_BF16>(name, reinterpret_cast<const __nv_bfloat16*>(h), M, F, ldh, nullptr, eps,
                                      q_rows, ldq, s_rows, q_cols_t, ldqt, s_cols, absmax_ws, st);
}

extern "C" int ff_swiglu_bwd_gemm_i8(const int8_t* A, int64_t lda, const int8_t* B, int64_t ldb,
                                     const float* scale_a, const uint16_t* gu, int64_t ldgu, const float* colmul,
                                     uint16_t* dgu, int64_t lddgu, int64_t M, int64_t F, int64_t K, float eps,
                                     int8_t* q_rows, int64_t ldq, float* s_rows, int8_t* q_cols_t, int64_t ldqt,
                                     float* s_cols, float* absmax_ws, void* stream) {
  using namespace ff;
  using namespace ff::gemm;
  const char* name = "ff_swiglu_bwd_gemm_i8";
  FF_REQUIRE(M >= 0 && F >= 1 && K >= 1, FF_ERR_INVALID_ARG, "%s: M=%lld F=%lld K=%lld", name, (long long)M,
             (long long)F, (long long)K);
  FF_REQUIRE(F % kSwigluFeat == 0, FF_ERR_UNSUPPORTED, "%s: F=%lld must be a multiple of %d", name, (long long)F,
             kSwigluFeat);
  FF_REQUIRE(q_rows || q_cols_t, FF_ERR_INVALID_ARG, "%s: nothing to do", name);
  if (M == 0) return FF_OK;
  FF_REQUIRE(A && B && gu && dgu, FF_ERR_INVALID_ARG, "%s: null pointer", name);
  FF_REQUIRE(lda >= K && ldb >= F && ldgu >= 2 * F && lddgu >= 2 * F, FF_ERR_INVALID_ARG, "%s: bad leading dims",
             name);
  FF_REQUIRE(aligned(A, 16) && aligned(B, 16) && lda % 16 == 0 && ldb % 16 == 0, FF_ERR_UNSUPPORTED,
             "%s: A/B need 16-byte alignment and lda/ldb multiples of 16", name);
  FF_REQUIRE(aligned(gu, 16) && aligned(dgu, 16) && ldgu % 8 == 0 && lddgu % 8 == 0, FF_ERR_UNSUPPORTED,
             "%s: gu/dgu need 16-byte alignment and leading dims multiples of 8", name);
  FF_REQUIRE(!colmul || aligned(colmul, 16), FF_ERR_UNSUPPORTED, "%s: colmul needs 16-byte alignment", name);
  FF_REQUIRE(M <= (int64_t)1 << 31 && 2 * F <= (int64_t)1 << 31 && K <= (int64_t)1 << 31, FF_ERR_UNSUPPORTED,
             "%s: dimension too large", name);
  int rc = check_dual_outputs(name, M, 2 * F, q_rows, ldq, s_rows, q_cols_t, ldqt, s_cols, absmax_ws);
  if (rc != FF_OK) return rc;
  const int max_pairs = max_pairs_current();
  FF_REQUIRE(max_pairs > 0, FF_ERR_UNSUPPORTED, "%s: the 2-CTA GEMM cannot be resident on this device", name);
  cudaStream_t st = as_stream(stream);
  FF_CUDA_TRY(cudaMemsetAsync(absmax_ws, 0, sizeof(float) * (size_t)(M + 2 * F), st), name);
  CUtensorMap ma, mb, md, mg;
  rc = make_map(&ma, A, M, K, lda, BM);
  if (rc) return rc;
  rc = make_map(&mb, B, K, F, ldb, BK);  // B is K x F row-major: read MN-major
  if (rc) return rc;
  // g/u loads and dg/du stores: boxes of one epilogue chunk (kSwbChunk features x 32 rows)
  rc = make_map_bf16(&md, dgu, M, 2 * F, lddgu, kSwbChunk, 32, CU_TENSOR_MAP_SWIZZLE_32B);
  if (rc) return rc;
  rc = make_map_bf16(&mg, gu, M, 2 * F, ldgu, kSwbChunk, 32, CU_TENSOR_MAP_SWIZZLE_32B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B);
  if (rc) return rc;
  EpiParams ep{};
  ep.scale_a = scale_a;
  ep.D = dgu;
  ep.ldd = lddgu;
  ep.M = M;
  ep.N = F;
  ep.vec = 1;
  ep.F = F;
  ep.row_amax = reinterpret_cast<uint32_t*>(absmax_ws);
  ep.col_amax = ep.row_amax + M;
  ep.g_in = reinterpret_cast<const __nv_bfloat16*>(gu);
  ep.ldg_in = ldgu;
  ep.colmul = colmul;
  const int t2m = (int)((M + 2 * C2_BM - 1) / (2 * C2_BM)), t2n = (int)((F + C2_BN - 1) / C2_BN);
  rc = launch_2cta<kOutSwigluBwd, true>(ma, mb, md, mg, K, t2m, t2n, ep, max_pairs, st);
  if (rc != FF_OK) return rc;
  return launch_pass_b<FF_DTYPE_BF16>(name, reinterpret_cast<const __nv_bfloat16*>(dgu), M, 2 * F, lddgu, colmul,
                                      eps, q_rows, ldq, s_rows, q_cols_t, ldqt, s_cols, absmax_ws, st);
}

extern "C" int ff_gelu_gemm_i8(const int8_t* A, int64_t lda, const int8_t* B, int64_t ldb, const float* scale_a,
                               const float* scale_b, const float* bias, uint16_t* u, int64_t ldu, uint16_t* h,
                               int64_t ldh, int64_t M, int64_t F, int64_t K, float eps, int variant, int8_t* q_rows,
                               int64_t ldq, float* s_rows, int8_t* q_cols_t, int64_t ldqt, float* s_cols,
                               float* absmax_ws, void* stream) {
  using namespace ff;
  using namespace ff::gemm;
  const char* name = "ff_gelu_gemm_i8";
  FF_REQUIRE(M >= 0 && F >= 1 && K >= 1 && variant >= 0 && variant < 64, FF_ERR_INVALID_ARG,
             "%s: M=%lld F=%lld K=%lld variant=%d", name, (long long)M, (long long)F, (long long)K, variant);
  FF_REQUIRE(F % 32 == 0, FF_ERR_UNSUPPORTED, "%s: F=%lld must be a multiple of 32", name, (long long)F);
  FF_REQUIRE(q_rows || q_cols_t, FF_ERR_INVALID_ARG, "%s: nothing to do", name);
  if (M == 0) return FF_OK;
  FF_REQUIRE(A && B && u && h, FF_ERR_INVALID_ARG, "%s: null pointer", name);
  FF_REQUIRE(lda >= K && ldb >= K && ldu >= F && ldh >= F, FF_ERR_INVALID_ARG, "%s: bad leading dims", name);
  FF_REQUIRE(aligned(A, 16) && aligned(B, 16) && lda % 16 == 0 && ldb % 16 == 0, FF_ERR_UNSUPPORTED,
             "%s: A/B need 16-byte alignment and lda/ldb multiples of 16", name);
  FF_REQUIRE(aligned(u, 16) && aligned(h, 16) && ldu % 8 == 0 && ldh % 8 == 0, FF_ERR_UNSUPPORTED,
             "%s: u/h need 16-byte alignment and leading dims multiples of 8", name);
  FF_REQUIRE((!scale_b || aligned(scale_b, 16)) && (!bias || aligned(bias, 16)), FF_ERR_UNSUPPORTED,
             "%s: scale_b/bias need 16-byte alignment", name);
  FF_REQUIRE(M <= (int64_t)1 << 31 && F <= (int64_t)1 << 31 && K <= (int64_t)1 << 31, FF_ERR_UNSUPPORTED,
             "%s: dimension too large", name);
  int rc = check_dual_outputs(name, M, F, q_rows, ldq, s_rows, q_cols_t, ldqt, s_cols, absmax_ws);
  if (rc != FF_OK) return rc;
  const int max_pairs = max_pairs_current();
  FF_REQUIRE(max_pairs > 0, FF_ERR_UNSUPPORTED, "%s: the 2-CTA GEMM cannot be resident on this device", name);
  cudaStream_t st = as_stream(stream);
  FF_CUDA_TRY(cudaMemsetAsync(absmax_ws, 0, sizeof(float) * (size_t)(M + F), st), name);
  CUtensorMap ma, mb, md, mh;
  rc = make_map(&ma, A, M, K, lda, BM);
  if (rc) return rc;
  rc = make_map(&mb, B, F, K, ldb, C2_BN_CTA);
  if (rc) return rc;
  // u and h stores: boxes of one epilogue chunk (kSwbChunk features x 32 rows)
  rc = make_map_bf16(&md, u, M, F, ldu, kSwbChunk, 32, CU_TENSOR_MAP_SWIZZLE_32B);
  if (rc) return rc;
  rc = make_map_bf16(&mh, h, M, F, ldh, kSwbChunk, 32, CU_TENSOR_MAP_SWIZZLE_32B);
  if (rc) return rc;
  EpiParams ep{};
  ep.scale_a = scale_a;
  ep.scale_b = scale_b;
  ep.bias = bias;
  ep.D = u;
  ep.ldd = ldu;
  ep.M = M;
  ep.N = F;
  ep.vec = 1;
  ep.h = reinterpret_cast<__nv_bfloat16*>(h);
  ep.ldh = ldh;
  ep.F = F;
  ep.row_amax = reinterpret_cast<uint32_t*>(absmax_ws);
  ep.col_amax = ep.row_amax + M;
  ep.act_variant = variant;
  const int t2m = (int)((M + 2 * C2_BM - 1) / (2 * C2_BM)), t2n = (int)((F + C2_BN - 1) / C2_BN);
  rc = launch_2cta<kOutGeluFwd, false>(ma, mb, md, mh, K, t2m, t2n, ep, max_pairs, st);
  if (rc != FF_OK) return rc;
  return launch_pass_b<FF_DTYPE_BF16>(name, reinterpret_cast<const __nv_bfloat16*>(h), M, F, ldh, nullptr, eps,
                                      q_rows, ldq, s_rows, q_cols_t, ldqt, s_cols, absmax_ws, st);
}

extern "C" int ff_gelu_bwd_gemm_i8(const int8_t* A, int64_t lda, const int8_t* B, int64_t ldb,
                                   const float* scale_a, const uint16_t* u, int64_t ldu, const float* colmul,
                                   uint16_t* du, int64_t lddu, int64_t M, int64_t F, int64_t K, float eps,
                                   int variant, int8_t* q_rows, int64_t ldq, float* s_rows, int8_t* q_cols_t,
                                   int64_t ldqt, float* s_cols, float* absmax_ws, void* stream) {
  using namespace ff;
  using namespace ff::gemm;
  const char* name = "ff_gelu_bwd_gemm_i8";
  FF_REQUIRE(M >= 0 && F >= 1 && K >= 1 && variant >= 0 && variant < 64, FF_ERR_INVALID_ARG,
             "%s: M=%lld F=%lld K=%lld variant=%d", name, (long long)M, (long long)F, (long long)K, variant);
  FF_REQUIRE(F % 32 == 0, FF_ERR_UNSUPPORTED, "%s: F=%lld must be a multiple of 32", name, (long long)F);
  FF_REQUIRE(q_rows || q_cols_t, FF_ERR_INVALID_ARG, "%s: nothing to do", name);
  if (M == 0) return FF_OK;
  FF_REQUIRE(A && B && u && du, FF_ERR_INVALID_ARG, "%s: null pointer", name);
  FF_REQUIRE(lda >= K && ldb >= F && ldu >= F && lddu >= F, FF_ERR_INVALID_ARG, "%s: bad leading dims", name);
  FF_REQUIRE(aligned(A, 16) && aligned(B, 16) && lda % 16 == 0 && ldb % 16 == 0, FF_ERR_UNSUPPORTED,
             "%s: A/B need 16-byte alignment and lda/ldb multiples of 16", name);
  FF_REQUIRE(aligned(u, 16) && aligned(du, 16) && ldu % 8 == 0 && lddu % 8 == 0, FF_ERR_UNSUPPORTED,
             "%s: u/du need 16-byte alignment and leading dims multiples of 8", name);
  FF_REQUIRE(!colmul || aligned(colmul, 16), FF_ERR_UNSUPPORTED, "%s: colmul needs 16-byte alignment", name);
  FF_REQUIRE(M <= (int64_t)1 << 31 && F <= (int64_t)1 << 31 && K <= (int64_t)1 << 31, FF_ERR_UNSUPPORTED,
             "%s: dimension too large", name);
  int rc = check_dual_outputs(name, M, F, q_rows, ldq, s_rows, q_cols_t, ldqt, s_cols, absmax_ws);
  if (rc != FF_OK) return rc;
  const int max_pairs = max_pairs_current();
  FF_REQUIRE(max_pairs > 0, FF_ERR_UNSUPPORTED, "%s: the 2-CTA GEMM cannot be resident on this device", name);
  cudaStream_t st = as_stream(stream);
  FF_CUDA_TRY(cudaMemsetAsync(absmax_ws, 0, sizeof(float) * (size_t)(M + F), st), name);
  CUtensorMap ma, mb, md;
  rc = make_map(&ma, A, M, K, lda, BM);
  if (rc) return rc;
  rc = make_map(&mb, B, K, F, ldb, BK);  // B is K x F row-major: read MN-major
  if (rc) return rc;
  // du stores and u loads: boxes of one epilogue chunk (kSwbChunk features x 32 rows)
  CUtensorMap mu;
  rc = make_map_bf16(&md, du, M, F, lddu, kSwbChunk, 32, CU_TENSOR_MAP_SWIZZLE_32B);
  if (rc) return rc;
  rc = make_map_bf16(&mu, u, M, F, ldu, kSwbChunk, 32, CU_TENSOR_MAP_SWIZZLE_32B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B);
  if (rc) return rc;
  EpiParams ep{};
  ep.scale_a = scale_a;
  ep.D = du;
  ep.ldd = lddu;
  ep.M = M;
  ep.N = F;
  ep.vec = 1;
  ep.F = F;
  ep.row_amax = reinterpret_cast<uint32_t*>(absmax_ws);
  ep.col_amax = ep.row_amax + M;
  ep.g_in = reinterpret_cast<const __nv_bfloat16*>(u);
  ep.ldg_in = ldu;
  ep.colmul = colmul;
  ep.act_variant = variant;
  const int t2m = (int)((M + 2 * C2_BM - 1) / (2 * C2_BM)), t2n = (int)((F + C2_BN - 1) / C2_BN);
  rc = launch_2cta<kOutGeluBwd, true>(ma, mb, md, mu, K, t2m, t2n, ep, max_pairs, st);
  if (rc != FF_OK) return rc;
  return launch_pass_b<FF_DTYPE_BF16>(name, reinterpret_cast<const __nv_bfloat16*>(du), M, F, lddu, colmul, eps,
                                      q_rows, ldq, s_rows, q_cols_t, ldqt, s_cols, absmax_ws, st);
}

extern "C" int ff_gemm_i8_kn(const int8_t* A, int64_t lda, const int8_t* B, int64_t ldb, const float* scale_a,
                             const float* scale_b, const float* bias, void* D, int64_t ldd, int out_kind, int64_t M,
                             int64_t N, int64_t K, void* stream) {
  return ff::gemm::gemm_dispatch<true>("ff_gemm_i8_kn", A, lda, B, ldb, scale_a, scale_b, bias, D, ldd, out_kind, M,
                                       N, K, stream);
}
