// dx_simt.cuh — CUDA-core fused linear with fp32 FFMA accumulation.
//
// Serves two cases the tensor-core kernels do not:
//   * fp32 inputs: the exact-fp32 path (no TF32 rounding of the operands),
//     needed for the fp32 tolerance of 1e-4;
//   * fp16/bf16 problems whose strides or pointers TMA cannot address
//     (rows not a multiple of 16 bytes), and K == 0.
// Each thread accumulates its outputs over k = 0..K-1 in order, so results
// are deterministic (and independent of the tile shape).  Tiles are BM x BN
// (16x32, 32x32 or 64x64) with 256 threads in a 16 x 16 grid; thread (ty, tx)
// owns rows ty + 16 i and columns tx + 16 j.  A gated form
// (two weight matrices, Y = act(X Wg + bg) * (X Wu + bu)) shares the tiling.
#pragma once

#include <type_traits>

#include "dx_epilogue.cuh"

namespace dx {

template <typename T, int BM, int BN, int BK>
__global__ void __launch_bounds__(256)
    simt_fused_linear_kernel(const T* __restrict__ X, const T* __restrict__ W,
                             const T* __restrict__ bias, const T* __restrict__ R,
                             T* __restrict__ Y, int M, int N, int K, long long ldx, long long ldw,
                             long long ldr, long long ldy, int act, float alpha) {
  using Tr = ElemTraits<T>;
  // K steps of BK; the next step's operands are loaded into registers while
  // the current step is multiplied from shared memory, so the global-memory
  // latency of a step overlaps the previous step's FFMAs.  Small tiles take
  // deep steps (few steps, each long enough to cover a load's latency).
  constexpr int TM = BM / 16;
  constexpr int TN = BN / 16;
  constexpr int A_PER = BM * BK / 256;  // X elements each thread stages per step
  constexpr int B_PER = BK * BN / 256;  // W elements each thread stages per step
  __shared__ float As[BK][BM + 1];
  __shared__ float Bs[BK][BN];
  const int tx = threadIdx.x & 15;
  const int ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * BM;
  const int n0 = blockIdx.x * BN;

  float ra[A_PER], rb[B_PER];
  auto load_step = [&](int k0) {
#pragma unroll
    for (int u = 0; u < A_PER; ++u) {
      const int idx = threadIdx.x + 256 * u;
      const int mm = idx / BK, kk = idx % BK;
      const int m = m0 + mm, k = k0 + kk;
      ra[u] = (m < M && k < K) ? Tr::to_float(X[m * ldx + k]) : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < B_PER; ++u) {
      const int idx = threadIdx.x + 256 * u;
      const int kk = idx / BN, nn = idx % BN;
      const int k = k0 + kk, n = n0 + nn;
      rb[u] = (k < K && n < N) ? Tr::to_float(W[k * ldw + n]) : 0.0f;
    }
  };

  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.0f;

  if (K > 0) load_step(0);
  for (int k0 = 0; k0 < K; k0 += BK) {
#pragma unroll
    for (int u = 0; u < A_PER; ++u) {
      const int idx = threadIdx.x + 256 * u;
      As[idx % BK][idx / BK] = ra[u];
    }
#pragma unroll
    for (int u = 0; u < B_PER; ++u) {
      const int idx = threadIdx.x + 256 * u;
      Bs[idx / BN][idx % BN] = rb[u];
    }
    __syncthreads();
    if (k0 + BK < K) load_step(k0 + BK);
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float a[TM], b[TN];
#pragma unroll
      for (int i = 0; i < TM; ++i) a[i] = As[kk][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < TN; ++j) b[j] = Bs[kk][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int m = m0 + ty + 16 * i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      const int n = n0 + tx + 16 * j;
      if (n >= N) continue;
      float v = alpha == 1.0f ? acc[i][j] : alpha * acc[i][j];
      if (bias != nullptr) v += Tr::to_float(bias[n]);
      v = act_apply<!std::is_same<T, float>::value>(v, act);
      if (R != nullptr) v += Tr::to_float(R[m * ldr + n]);
      Y[m * ldy + n] = Tr::from_float(v);
    }
  }
}

// Gated form: Y = act(X Wg + bg) * (X Wu + bu), same tiling, two accumulator
// sets (gate and up) fed by one X tile.
template <typename T, int BM, int BN>
__global__ void __launch_bounds__(256)
    simt_gated_linear_kernel(const T* __restrict__ X, const T* __restrict__ Wg,
                             const T* __restrict__ Wu, const T* __restrict__ bg,
                             const T* __restrict__ bu, T* __restrict__ Y, int M, int N, int K,
                             long long ldx, long long ldwg, long long ldwu, long long ldy, int act) {
  using Tr = ElemTraits<T>;
  constexpr int BK = 16;
  constexpr int TM = BM / 16;
  constexpr int TN = BN / 16;
  __shared__ float As[BK][BM + 1];
  __shared__ float Gs[BK][BN];
  __shared__ float Us[BK][BN];
  const int tx = threadIdx.x & 15;
  const int ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * BM;
  const int n0 = blockIdx.x * BN;

  float ag[TM][TN], au[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) ag[i][j] = au[i][j] = 0.0f;

  for (int k0 = 0; k0 < K; k0 += BK) {
    for (int idx = threadIdx.x; idx < BM * BK; idx += 256) {
      const int mm = idx / BK, kk = idx % BK;
      const int m = m0 + mm, k = k0 + kk;
      As[kk][mm] = (m < M && k < K) ? Tr::to_float(X[m * ldx + k]) : 0.0f;
    }
    for (int idx = threadIdx.x; idx < BK * BN; idx += 256) {
      const int kk = idx / BN, nn = idx % BN;
      const int k = k0 + kk, n = n0 + nn;
      const bool in = k < K && n < N;
      Gs[kk][nn] = in ? Tr::to_float(Wg[k * ldwg + n]) : 0.0f;
      Us[kk][nn] = in ? Tr::to_float(Wu[k * ldwu + n]) : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float a[TM], g[TN], u[TN];
#pragma unroll
      for (int i = 0; i < TM; ++i) a[i] = As[kk][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < TN; ++j) {
        g[j] = Gs[kk][tx + 16 * j];
        u[j] = Us[kk][tx + 16 * j];
      }
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) {
          ag[i][j] = fmaf(a[i], g[j], ag[i][j]);
          au[i][j] = fmaf(a[i], u[j], au[i][j]);
        }
    }
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int m = m0 + ty + 16 * i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      const int n = n0 + tx + 16 * j;
      if (n >= N) continue;
      float gv = ag[i][j], uv = au[i][j];
      if (bg != nullptr) gv += Tr::to_float(bg[n]);
      if (bu != nullptr) uv += Tr::to_float(bu[n]);
      Y[m * ldy + n] = Tr::from_float(act_apply<!std::is_same<T, float>::value>(gv, act) * uv);
    }
  }
}

}  // namespace dx
