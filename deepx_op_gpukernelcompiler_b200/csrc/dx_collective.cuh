// dx_collective.cuh — the reduction of a row-parallel linear over ranks.
//
// A row-parallel GEMM (the second layer of the MLP chain, with its K
// dimension sharded over ranks) leaves every rank with a partial Y in its own
// peer-mapped buffer.  Every rank then runs this kernel on its own slab of
// rows: it reads the slab from all `world` partial buffers (peer loads over
// NVLink, 16 B per thread, consecutive threads on consecutive columns), adds
// them in rank order (fixed, so results do not depend on timing), adds bias
// and residual once, rounds, and writes the finished rows into every rank's
// output buffer (peer stores) — reduce-scatter and all-gather in one pass.
#pragma once

#include "dx_epilogue.cuh"

namespace dx {

struct RankPtrs {
  void* p[8];
};

// P:    every rank's partial buffer, global rows, pitch ldp
// R:    [rows][ldr] residual (global rows), or nullptr; bias [N] or nullptr
// Y:    every rank's output buffer, global rows, pitch ldy
template <typename T>
__global__ void __launch_bounds__(256)
    reduce_broadcast_kernel(RankPtrs P, int world, int rank, int rows_per_rank, int N,
                            long long ldp, const T* __restrict__ bias, const T* __restrict__ R,
                            long long ldr, RankPtrs Y, long long ldy) {
  using Tr = ElemTraits<T>;
  const int groups = N / 8;  // 8 columns (16 bytes) per thread-step
  const long long total = static_cast<long long>(rows_per_rank) * groups;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += stride) {
    const int r = static_cast<int>(i / groups);
    const int c8 = static_cast<int>(i - static_cast<long long>(r) * groups) * 8;
    const long long row = static_cast<long long>(rank) * rows_per_rank + r;
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
    uint4 part[8];
#pragma unroll
    for (int src = 0; src < 8; ++src)
      if (src < world)
        part[src] = __ldcs(reinterpret_cast<const uint4*>(static_cast<const T*>(P.p[src]) +
                                                          row * ldp + c8));
#pragma unroll
    for (int src = 0; src < 8; ++src) {
      if (src >= world) break;
      const uint4 w = part[src];
      const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float2 f = Tr::unpack2(wv[h]);
        acc[2 * h] += f.x;
        acc[2 * h + 1] += f.y;
      }
    }
    if (bias != nullptr) {
      const uint4 w = __ldg(reinterpret_cast<const uint4*>(bias + c8));
      const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float2 f = Tr::unpack2(wv[h]);
        acc[2 * h] += f.x;
        acc[2 * h + 1] += f.y;
      }
    }
    if (R != nullptr) {
      const uint4 w = __ldcs(reinterpret_cast<const uint4*>(R + row * ldr + c8));
      const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float2 f = Tr::unpack2(wv[h]);
        acc[2 * h] += f.x;
        acc[2 * h + 1] += f.y;
      }
    }
    uint4 out;
    out.x = Tr::pack2(acc[0], acc[1]);
    out.y = Tr::pack2(acc[2], acc[3]);
    out.z = Tr::pack2(acc[4], acc[5]);
    out.w = Tr::pack2(acc[6], acc[7]);
    for (int d = 0; d < world; ++d)
      *reinterpret_cast<uint4*>(static_cast<T*>(Y.p[d]) + row * ldy + c8) = out;
  }
  __threadfence_system();
}

}  // namespace dx
