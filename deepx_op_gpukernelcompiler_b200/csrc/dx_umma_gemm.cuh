// dx_umma_gemm.cuh — persistent tcgen05 GEMM with the fused linear epilogue:
//   Y[M,N] = act(X[M,K] @ W[K,N] + bias[N]) (+ R[M,N]),  fp16/bf16 in and out,
//   fp32 accumulation in TMEM.
//
// This replaces the reference's per-tile K loop + epilogue
// (kernel_triton.py:47-67, kernel_tilelang.py:36-53) with a B200 design:
//   * one CTA per SM, looping over 128 x BN output tiles (static schedule,
//     M-fastest inside groups of `group_m` m-tiles so a panel of X stays in
//     L2 while all of W streams past it);
//   * warp 0: TMA producer.  X tiles [128 x 64] (K-major) and W tiles
//     [64 x BN] (N-major, i.e. W exactly as it sits in memory) land in a
//     STAGES-deep ring of 128-byte-swizzled shared-memory buffers;
//   * warp 1: TMEM allocator and the single thread that issues
//     tcgen05.mma (M=128, N=BN, K=16) into one of two TMEM accumulators;
//   * warps 2-5: epilogue.  Each warp owns the 32 TMEM lanes (= tile rows) it
//     may address, pulls 32 columns at a time with tcgen05.ld, adds bias,
//     applies the activation, adds the residual (TMA-loaded into the same
//     staging buffer), converts and TMA-stores.  The output tile crosses HBM
//     exactly once; the next tile's main loop runs in the other accumulator
//     meanwhile.
// Every mbarrier wait is bounded (dx_ptx.cuh); a timed-out CTA drains its
// copies in flight, frees TMEM and exits with the device status bit set.
#pragma once

#include "dx_epilogue.cuh"
#include "dx_ptx.cuh"

namespace dx {

struct UmmaParams {
  int M, N, K;
  int m_tiles, n_tiles, k_blocks, num_tiles;
  int group_m;       // m-tiles per raster group
  const void* bias;  // N elements, or nullptr
  int act;
  int has_residual;
};

template <int BN>
struct UmmaShape {
  static constexpr int BM = 128;
  static constexpr int BK = 64;  // 64 x 16-bit = one 128-byte swizzle row
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BK * BN * 2;
  static constexpr int B_BOX_BYTES = BK * 64 * 2;  // one [64 k x 64 n] TMA box
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (BN == 256) ? 4 : 6;
  static constexpr int EPI_WARPS = 4;
  static constexpr int EPI_BUF_BYTES = 32 * 32 * 2;  // [32 rows x 32 cols] 16-bit
  static constexpr int TMEM_COLS = 2 * BN;           // two fp32 accumulators
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + STAGES * A_BYTES;
  static constexpr int OFF_EPI = OFF_B + STAGES * B_BYTES;
  static constexpr int OFF_BAR = OFF_EPI + EPI_WARPS * 2 * EPI_BUF_BYTES;
  // full[STAGES], empty[STAGES], tmem_full[2], tmem_empty[2],
  // residual[EPI_WARPS][2], drain
  static constexpr int BAR_FULL = 0;
  static constexpr int BAR_EMPTY = STAGES;
  static constexpr int BAR_TFULL = 2 * STAGES;
  static constexpr int BAR_TEMPTY = 2 * STAGES + 2;
  static constexpr int BAR_RES = 2 * STAGES + 4;
  static constexpr int BAR_DRAIN = BAR_RES + 2 * EPI_WARPS;
  static constexpr int NUM_BARS = BAR_DRAIN + 1;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;  // tmem base, abort flag
  static constexpr int SMEM_BYTES = 1024 + OFF_MISC + 16;
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
  static_assert(BN % 64 == 0 && BN >= 64 && BN <= 256, "UMMA N");
};

__device__ __forceinline__ void umma_tile_coords(const UmmaParams& p, int t, int& mb, int& nb) {
  const int per_group = p.group_m * p.n_tiles;
  const int g = t / per_group;
  const int r = t - g * per_group;
  const int m_first = g * p.group_m;
  const int gm = min(p.group_m, p.m_tiles - m_first);
  mb = m_first + r % gm;
  nb = r / gm;
}

template <int BN, typename T>
__global__ void __launch_bounds__(UmmaShape<BN>::THREADS, 1)
    umma_fused_linear_kernel(const __grid_constant__ CUtensorMap tmA,
                             const __grid_constant__ CUtensorMap tmB,
                             const __grid_constant__ CUtensorMap tmY,
                             const __grid_constant__ CUtensorMap tmR, const UmmaParams p) {
  using S = UmmaShape<BN>;
  using Tr = ElemTraits<T>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t base = (raw_u32 + 1023u) & ~1023u;
  uint8_t* const base_ptr = smem_raw + (base - raw_u32);

  const uint32_t sA = base + S::OFF_A;
  const uint32_t sB = base + S::OFF_B;
  const uint32_t bars = base + S::OFF_BAR;
  uint32_t* const tmem_word = reinterpret_cast<uint32_t*>(base_ptr + S::OFF_MISC);
  volatile int* const abort_flag = reinterpret_cast<volatile int*>(base_ptr + S::OFF_MISC + 4);
  auto bar = [bars](int i) { return bars + 8u * static_cast<uint32_t>(i); };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::STAGES; ++s) {
      mbar_init(bar(S::BAR_FULL + s), 1);
      mbar_init(bar(S::BAR_EMPTY + s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar(S::BAR_TFULL + b), 1);
      mbar_init(bar(S::BAR_TEMPTY + b), S::EPI_WARPS);
    }
    for (int i = 0; i < 2 * S::EPI_WARPS; ++i) mbar_init(bar(S::BAR_RES + i), 1);
    mbar_init(bar(S::BAR_DRAIN), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmY);
    if (p.has_residual) tma_prefetch_desc(&tmR);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_word), S::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_word;

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0, issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < p.num_tiles; t += gridDim.x) {
        int mb, nb;
        umma_tile_coords(p, t, mb, nb);
        const int m0 = mb * S::BM, n0 = nb * BN;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(bar(S::BAR_EMPTY + s), ph ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t fb = bar(S::BAR_FULL + s);
          mbar_arrive_expect_tx(fb, S::STAGE_BYTES);
          tma_load_2d(&tmA, sA + s * S::A_BYTES, fb, kb * S::BK, m0);
#pragma unroll
          for (int j = 0; j < BN / 64; ++j)
            tma_load_2d(&tmB, sB + s * S::B_BYTES + j * S::B_BOX_BYTES, fb, n0 + 64 * j,
                        kb * S::BK);
          ++issued;
          if (++s == S::STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      // Loads still in flight must land before this CTA's shared memory is
      // released.  On the normal path these waits return at once.
      const uint32_t n_drain = issued < (uint32_t)S::STAGES ? issued : (uint32_t)S::STAGES;
      for (uint32_t i = issued - n_drain; i < issued; ++i)
        mbar_wait_drain(bar(S::BAR_FULL + (int)(i % S::STAGES)), (i / S::STAGES) & 1u);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(Tr::kIsBf16, 128, BN, false, true);
      int s = 0, local = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < p.num_tiles; t += gridDim.x, ++local) {
        const int b = local & 1;
        const uint32_t use_ph = (static_cast<uint32_t>(local) >> 1) & 1u;
        if (!mbar_wait(bar(S::BAR_TEMPTY + b), use_ph ^ 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(b * BN);
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(bar(S::BAR_FULL + s), ph, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // X tile: K-major, 8-row groups 1024 B apart; +32 B per K=16 step.
          const uint64_t ad = smem_desc_sw128(sA + s * S::A_BYTES, 16, 1024);
          // W tile: N-major, 64-wide n groups one box (8 KB) apart, 8-row k
          // groups 1024 B apart; +2048 B per K=16 step.
          const uint64_t bd = smem_desc_sw128(sB + s * S::B_BYTES, S::B_BOX_BYTES, 1024);
#pragma unroll
          for (int k = 0; k < S::BK / 16; ++k)
            umma_f16(d_tmem, ad + 2ull * k, bd + 128ull * k, idesc, (kb | k) != 0 ? 1u : 0u);
          umma_commit(bar(S::BAR_EMPTY + s));
          if (++s == S::STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (ok) umma_commit(bar(S::BAR_TFULL + b));
      }
      // Every MMA issued so far completes before TMEM can be freed.
      umma_commit(bar(S::BAR_DRAIN));
      mbar_wait_drain(bar(S::BAR_DRAIN), 0);
    }
    __syncwarp();
  } else {
    // --------------------------------------------------------- epilogue
    const int e = warp - 2;  // epilogue warp index 0..3
    const int q = warp & 3;  // TMEM lane quarter this warp may address
    const T* const bias = static_cast<const T*>(p.bias);
    const bool bias_vec_ok = bias != nullptr && (reinterpret_cast<uintptr_t>(bias) & 15u) == 0;
    const uint32_t ebuf0 = base + S::OFF_EPI + e * 2 * S::EPI_BUF_BYTES;
    uint8_t* const ebuf_ptr0 = base_ptr + S::OFF_EPI + e * 2 * S::EPI_BUF_BYTES;
    const uint32_t row_off = static_cast<uint32_t>(lane) * 64u;
    const uint32_t row_sw = (static_cast<uint32_t>(lane) >> 1) & 3u;  // 64-byte swizzle phase
    uint32_t it = 0;
    int local = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < p.num_tiles; t += gridDim.x, ++local) {
      const int b = local & 1;
      const uint32_t use_ph = (static_cast<uint32_t>(local) >> 1) & 1u;
      if (!mbar_wait(bar(S::BAR_TFULL + b), use_ph, abort_flag)) break;
      tc_fence_after();
      int mb, nb;
      umma_tile_coords(p, t, mb, nb);
      const int m0 = mb * S::BM, n0 = nb * BN;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c, ++it) {
        const int buf = it & 1;
        const uint32_t ebuf = ebuf0 + buf * S::EPI_BUF_BYTES;
        uint8_t* const ebp = ebuf_ptr0 + buf * S::EPI_BUF_BYTES;
        const int n_c = n0 + 32 * c;
        // The store issued two chunks ago from this buffer must have read it.
        if (lane == 0) bulk_wait_group_read<1>();
        __syncwarp();
        const uint32_t rbar = bar(S::BAR_RES + e * 2 + buf);
        if (p.has_residual && lane == 0) {
          mbar_arrive_expect_tx(rbar, S::EPI_BUF_BYTES);
          tma_load_2d(&tmR, ebuf, rbar, n_c, m0 + q * 32);
        }
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + static_cast<uint32_t>(b * BN + 32 * c) +
                               (static_cast<uint32_t>(q * 32) << 16),
                           r);
        tmem_wait_ld();
        if (c == BN / 32 - 1) {
          // Accumulator fully read: hand it back to the MMA warp.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(S::BAR_TEMPTY + b));
        }
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        if (bias != nullptr) {
          if (bias_vec_ok && n_c + 32 <= p.N) {
            const uint4* bp = reinterpret_cast<const uint4*>(bias + n_c);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint4 w = __ldg(bp + j);
              const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
              for (int h = 0; h < 4; ++h) {
                const float2 f = Tr::unpack2(wv[h]);
                v[8 * j + 2 * h] += f.x;
                v[8 * j + 2 * h + 1] += f.y;
              }
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (n_c + j < p.N) v[j] += Tr::to_float(bias[n_c + j]);
          }
        }
        if (p.act != kActNone) {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = act_apply(v[j], p.act);
        }
        if (p.has_residual) {
          if (!mbar_wait(rbar, (it >> 1) & 1u, abort_flag)) {
            mbar_wait_drain(rbar, (it >> 1) & 1u);  // the load still lands here
            ok = false;
            break;
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint4 w =
                *reinterpret_cast<const uint4*>(ebp + row_off + ((static_cast<uint32_t>(j) ^ row_sw) << 4));
            const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int h = 0; h < 4; ++h) {
              const float2 f = Tr::unpack2(wv[h]);
              v[8 * j + 2 * h] += f.x;
              v[8 * j + 2 * h + 1] += f.y;
            }
          }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint4 w;
          w.x = Tr::pack2(v[8 * j + 0], v[8 * j + 1]);
          w.y = Tr::pack2(v[8 * j + 2], v[8 * j + 3]);
          w.z = Tr::pack2(v[8 * j + 4], v[8 * j + 5]);
          w.w = Tr::pack2(v[8 * j + 6], v[8 * j + 7]);
          *reinterpret_cast<uint4*>(ebp + row_off + ((static_cast<uint32_t>(j) ^ row_sw) << 4)) = w;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmY, ebuf, n_c, m0 + q * 32);
          bulk_commit_group();
        }
      }
    }
    if (lane == 0) bulk_wait_group<0>();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, S::TMEM_COLS);
  }
}

}  // namespace dx
