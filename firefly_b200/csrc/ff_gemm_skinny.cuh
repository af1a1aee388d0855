// ff_gemm_skinny.cuh — int8 GEMM for skinny A (M <= 128 rows): stream-K over every SM.
//
//   acc[m, n] = sum_k A[m, k] * B[n, k],  D[m, n] = epilogue(acc)   (the ff_gemm_i8 contract)
//
// With few rows of A the GEMM is a stream over B (N x K bytes), so the work is laid out for
// HBM bandwidth, not for tensor throughput:
//
// * Operands swapped on the tensor core: a 128-row tile of B is the MMA's M side and the M
//   (padded to MP = 16, 32, 64 or 128) rows of A its N side, tcgen05.mma kind::i8 128 x MP x 32,
//   so no tensor-core row or smem byte is spent on padding A up to 128 rows.
// * Stream-K: the (n-tile, 128-byte k-block) iterations of the whole problem are cut into one
//   contiguous range per CTA (grid = SM count), so every SM streams the same number of B bytes
//   through a 6 to 11 stage TMA ring (no multicast).
// * A tile whose k-range is split between CTAs is combined in a workspace of int32 partial
//   sums: every contributor adds its partial with red.global.add (exact: int32 addition is
//   associative), then bumps the tile's counter; the contributor that arrives last applies
//   the epilogue to the total and writes zeros back, so the workspace is all zeros again after
//   every call and no CTA ever waits for another.
//
// Warp roles as in gemm_i8_kernel: warp 0 TMA producer, warp 1 TMEM allocation and MMA issue,
// warps 2-5 epilogue (TMEM lane quarter = warp % 4).  Two accumulators of MP columns let the
// epilogue of one range overlap the MMAs of the next.  All waits are time-bounded.
//
// Included by ff_gemm_i8.cuh after its device helpers and before its host dispatch.
#pragma once

namespace ff {
namespace gemm {

constexpr int SK_BN = 128;  // rows of B per tile (the MMA's M)
__host__ __device__ constexpr int sk_stage_bytes(int mp) { return SK_BN * BK + mp * BK; }
__host__ __device__ constexpr int sk_stages(int mp) {
  return (200 * 1024) / sk_stage_bytes(mp) > 12 ? 12 : (200 * 1024) / sk_stage_bytes(mp);
}
__host__ __device__ constexpr int sk_smem_bytes(int mp) {
  return sk_stages(mp) * sk_stage_bytes(mp) + 1024 /*align*/ + 512 /*barriers, flags*/ + mp * 4 /*scale_a*/;
}
__host__ __device__ constexpr int sk_tmem_cols(int mp) { return 2 * mp < 32 ? 32 : 2 * mp; }
// workspace: per tile MP x 128 int32 partial sums, then one uint32 counter per tile
inline int64_t sk_ws_bytes(int64_t tiles, int mp) { return tiles * mp * SK_BN * 4 + tiles * 4; }
inline int sk_mp(int64_t M) { return M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : 128; }

// the CTA whose k-iteration range holds iteration i (ranges [c*total/G, (c+1)*total/G))
__device__ __forceinline__ int64_t sk_owner(int64_t i, int64_t total, int64_t G) { return ((i + 1) * G + total - 1) / total - 1; }

// epilogue of W values of one column n (rows m0 + j < M) from their int32 totals, in the
// ff_gemm_i8 op order; the bf16 accumulate variant reads all W old values before writing
template <int OUT, int W>
__device__ __forceinline__ void sk_store(const EpiParams& ep, int m0, int64_t n, const uint32_t* acc,
                                         const float* sa, float sb, float bias) {
  const int nm = (int)min64(W, ep.M - m0);
  if constexpr (OUT == FF_OUT_S32) {
#pragma unroll
    for (int j = 0; j < W; ++j)
      if (j < nm) reinterpret_cast<uint32_t*>(ep.D)[(int64_t)(m0 + j) * ep.ldd + n] = acc[j];
  } else {
    float t[W];
#pragma unroll
    for (int j = 0; j < W; ++j) {
      t[j] = __int2float_rn((int)acc[j]);
      if (ep.scale_a) t[j] = __fmul_rn(t[j], sa[m0 + j]);
      if (ep.scale_b) t[j] = __fmul_rn(t[j], sb);
      if (ep.bias) t[j] = __fadd_rn(t[j], bias);
    }
    if constexpr (OUT == FF_OUT_F32) {
#pragma unroll
      for (int j = 0; j < W; ++j)
        if (j < nm) reinterpret_cast<float*>(ep.D)[(int64_t)(m0 + j) * ep.ldd + n] = t[j];
    } else {
      __nv_bfloat16* d = reinterpret_cast<__nv_bfloat16*>(ep.D) + (int64_t)m0 * ep.ldd + n;
      if constexpr (OUT == FF_OUT_BF16_ACCUM) {
        float old[W];
#pragma unroll
        for (int j = 0; j < W; ++j) old[j] = j < nm ? __bfloat162float(d[(int64_t)j * ep.ldd]) : 0.f;
#pragma unroll
        for (int j = 0; j < W; ++j)
          if (j < nm)
            d[(int64_t)j * ep.ldd] =
                __float2bfloat16_rn(__fadd_rn(old[j], __bfloat162float(__float2bfloat16_rn(t[j]))));
      } else {
#pragma unroll
        for (int j = 0; j < W; ++j)
          if (j < nm) d[(int64_t)j * ep.ldd] = __float2bfloat16_rn(t[j]);
      }
    }
  }
}

template <int OUT, int MP>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_i8_skinny_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                          int64_t K, int tiles, EpiParams ep, int32_t* ws, uint32_t* counters) {
  constexpr int STAGES_ = sk_stages(MP);
  constexpr int A_BYTES_ = MP * BK, B_BYTES_ = SK_BN * BK;
  constexpr int TMEM_COLS_ = sk_tmem_cols(MP);
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t pad = (1024u - (raw_addr & 1023u)) & 1023u;
  uint8_t* smem = smem_raw + pad;
  const uint32_t sbase = raw_addr + pad;
  const uint32_t sB = sbase;                         // STAGES_ x 16 KiB (1024-aligned)
  const uint32_t sA = sbase + STAGES_ * B_BYTES_;    // STAGES_ x MP*128 B (multiples of 2 KiB)
  uint8_t* ctrl = smem + STAGES_ * (A_BYTES_ + B_BYTES_);
  const uint32_t cbase = sbase + STAGES_ * (A_BYTES_ + B_BYTES_);
  auto full_bar = [&](int s) { return cbase + 8u * s; };
  auto empty_bar = [&](int s) { return cbase + 8u * (STAGES_ + s); };
  auto tfull_bar = [&](int a) { return cbase + 8u * (2 * STAGES_ + a); };
  auto tempty_bar = [&](int a) { return cbase + 8u * (2 * STAGES_ + ACC_STAGES + a); };
  const uint32_t drain = cbase + 8u * (2 * STAGES_ + 2 * ACC_STAGES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ctrl + 8 * (2 * STAGES_ + 2 * ACC_STAGES + 1));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(ctrl + 8 * (2 * STAGES_ + 2 * ACC_STAGES + 1) + 4);
  volatile int* last_flag = reinterpret_cast<volatile int*>(ctrl + 8 * (2 * STAGES_ + 2 * ACC_STAGES + 1) + 8);
  float* s_sa = reinterpret_cast<float*>(ctrl + 512);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_kb = (int)((K + BK - 1) / BK);
  const int64_t total = (int64_t)tiles * num_kb;
  const int64_t G = gridDim.x;
  const int64_t beg = (int64_t)blockIdx.x * total / G, end = ((int64_t)blockIdx.x + 1) * total / G;

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
  if (warp >= 2) {  // the row scales of A, read by the epilogue for every value
    for (int j = threadIdx.x - 64; j < MP; j += 128)
      s_sa[j] = (OUT != FF_OUT_S32 && ep.scale_a && j < ep.M) ? __ldg(ep.scale_a + j) : 1.f;
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
      uint32_t phase = 0, used = 0, last_phase = 0;
      bool ok = true;
      for (int64_t it = beg; it < end && ok;) {
        const int tile = (int)(it / num_kb);
        const int lo = (int)(it - (int64_t)tile * num_kb);
        const int hi = (int)min64(num_kb, lo + (end - it));
        for (int kb = lo; kb < hi; ++kb) {
          if (!wait_bar(empty_bar(stage), phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(full_bar(stage), A_BYTES_ + B_BYTES_);
          tma_load_2d(sB + stage * B_BYTES_, &tmB, kb * BK, tile * SK_BN, full_bar(stage));
          tma_load_2d(sA + stage * A_BYTES_, &tmA, kb * BK, 0, full_bar(stage));
          used |= 1u << stage;
          last_phase = (last_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES_) {
            stage = 0;
            phase ^= 1u;
          }
        }
        it += hi - lo;
      }
      for (int s = 0; s < STAGES_; ++s)
        if (used & (1u << s)) drain_bar(full_bar(s), (last_phase >> s) & 1u);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_i8(SK_BN, MP);
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int64_t it = beg; it < end && ok;) {
        const int tile = (int)(it / num_kb);
        const int lo = (int)(it - (int64_t)tile * num_kb);
        const int hi = (int)min64(num_kb, lo + (end - it));
        if (!wait_bar(tempty_bar(acc), acc_phase ^ 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * MP);
        for (int kb = lo; kb < hi; ++kb) {
          if (!wait_bar(full_bar(stage), phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t b0 = sB + stage * B_BYTES_, a0 = sA + stage * A_BYTES_;
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; ++k)
            tc_mma_i8(d_tmem, smem_desc_k_sw128(b0 + k * UMMA_K), smem_desc_k_sw128(a0 + k * UMMA_K), idesc,
                      (kb != lo || k != 0) ? 1u : 0u);
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
        it += hi - lo;
      }
      tc_commit(drain);
      drain_bar(drain, 0);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue (warps 2-5)
    const int lg = warp & 3;
    const int nl = lg * 32 + lane;  // this thread's row of the B tile = its TMEM lane
    const bool first = threadIdx.x == 64;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int64_t it = beg; it < end;) {
      const int tile = (int)(it / num_kb);
      const int lo = (int)(it - (int64_t)tile * num_kb);
      const int hi = (int)min64(num_kb, lo + (end - it));
      it += hi - lo;
      const int64_t n = (int64_t)tile * SK_BN + nl;
      const bool nvalid = n < ep.N;
      float sb = 1.f, bias = 0.f;
      if constexpr (OUT != FF_OUT_S32) {
        if (ep.scale_b && nvalid) sb = __ldg(ep.scale_b + n);
        if (ep.bias && nvalid) bias = __ldg(ep.bias + n);
      }
      const int64_t it0 = (int64_t)tile * num_kb;
      const int64_t contributors = sk_owner(it0 + num_kb - 1, total, G) - sk_owner(it0, total, G) + 1;
      if (!wait_bar(tfull_bar(acc), acc_phase, abort_flag)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + ((uint32_t)(lg * 32) << 16) + (uint32_t)(acc * MP);
      int32_t* wt = ws + (int64_t)tile * MP * SK_BN + nl;  // this thread's column of the tile's partial sums
#pragma unroll 1
      for (int c = 0; c < MP; c += 32) {
        uint32_t r[32];
        if constexpr (MP == 16) {
          tmem_ld16(tbase, r);
        } else {
          tmem_ld32(tbase + c, r);
        }
        tmem_wait_ld();
        constexpr int W = MP == 16 ? 16 : 32;
        if (contributors == 1) {
          if (nvalid && c < ep.M) sk_store<OUT, W>(ep, c, n, r, s_sa, sb, bias);
        } else {
#pragma unroll
          for (int j = 0; j < W; ++j) atomicAdd(wt + (int64_t)(c + j) * SK_BN, (int)r[j]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty_bar(acc));
      if (++acc == ACC_STAGES) {
        acc = 0;
        acc_phase ^= 1u;
      }
      if (contributors > 1) {
        // every epilogue thread's partial sums are issued: count this CTA in, and the last
        // contributor finishes the tile
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (first) {
          __threadfence();
          const uint32_t old = atomicAdd(counters + tile, 1u);
          *last_flag = (old == (uint32_t)(contributors - 1)) ? 1 : 0;
          __threadfence();
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (*last_flag) {
          // the total: 16 or 32 loads in flight at a time, then zeros written back
          constexpr int W = MP == 16 ? 16 : 32;
#pragma unroll 1
          for (int c = 0; c < MP; c += W) {
            uint32_t v[W];
#pragma unroll
            for (int j = 0; j < W; ++j) v[j] = (uint32_t)__ldcg(wt + (int64_t)(c + j) * SK_BN);
#pragma unroll
            for (int j = 0; j < W; ++j) wt[(int64_t)(c + j) * SK_BN] = 0;
            if (nvalid && c < ep.M) sk_store<OUT, W>(ep, c, n, v, s_sa, sb, bias);
          }
          if (first) counters[tile] = 0u;
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");  // last_flag is read before it is rewritten
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

template <int OUT, int MP>
inline int launch_skinny(const CUtensorMap& ma, const CUtensorMap& mb, int64_t K, int tiles, const EpiParams& ep,
                         int grid, int32_t* ws, uint32_t* counters, cudaStream_t st) {
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    FF_CUDA_TRY(cudaFuncSetAttribute(gemm_i8_skinny_kernel<OUT, MP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     sk_smem_bytes(MP)),
                "ff_gemm_i8 skinny smem attribute");
    attr_set[dev] = true;
  }
  gemm_i8_skinny_kernel<OUT, MP><<<grid, NUM_THREADS, sk_smem_bytes(MP), st>>>(ma, mb, K, tiles, ep, ws, counters);
  return check_launch("ff_gemm_i8 (skinny)");
}

template <int OUT>
inline int launch_skinny_mp(int mp, const CUtensorMap& ma, const CUtensorMap& mb, int64_t K, int tiles,
                            const EpiParams& ep, int grid, int32_t* ws, uint32_t* counters, cudaStream_t st) {
  switch (mp) {
    case 16: return launch_skinny<OUT, 16>(ma, mb, K, tiles, ep, grid, ws, counters, st);
    case 32: return launch_skinny<OUT, 32>(ma, mb, K, tiles, ep, grid, ws, counters, st);
    case 64: return launch_skinny<OUT, 64>(ma, mb, K, tiles, ep, grid, ws, counters, st);
    default: return launch_skinny<OUT, 128>(ma, mb, K, tiles, ep, grid, ws, counters, st);
  }
}

}  // namespace gemm
}  // namespace ff
