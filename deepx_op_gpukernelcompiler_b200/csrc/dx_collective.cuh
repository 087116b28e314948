// dx_collective.cuh — the reduction of a row-parallel linear over ranks.
//
// A row-parallel GEMM (the output projection of the MLP or gated FFN chain,
// its K dimension sharded over ranks) leaves every rank with a partial Y in its own
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
// Sums one 16-byte column group of one row over the ranks' partials (all
// loads issued before the adds) and adds bias and residual.
template <typename T>
__device__ __forceinline__ void rb_load(const RankPtrs& P, int world, long long off, uint4 (&part)[8]) {
#pragma unroll
  for (int src = 0; src < 8; ++src)
    if (src < world) part[src] = __ldcs(reinterpret_cast<const uint4*>(static_cast<const T*>(P.p[src]) + off));
}

template <typename T>
__device__ __forceinline__ uint4 rb_finish(const uint4 (&part)[8], int world, const T* bias,
                                          const T* R, long long roff, int c8) {
  using Tr = ElemTraits<T>;
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
  auto add = [&acc](const uint4& w) {
    const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const float2 f = Tr::unpack2(wv[h]);
      acc[2 * h] += f.x;
      acc[2 * h + 1] += f.y;
    }
  };
#pragma unroll
  for (int src = 0; src < 8; ++src)
    if (src < world) add(part[src]);  // rank order
  if (bias != nullptr) add(__ldg(reinterpret_cast<const uint4*>(bias + c8)));
  if (R != nullptr) add(__ldcs(reinterpret_cast<const uint4*>(R + roff)));
  uint4 out;
  out.x = Tr::pack2(acc[0], acc[1]);
  out.y = Tr::pack2(acc[2], acc[3]);
  out.z = Tr::pack2(acc[4], acc[5]);
  out.w = Tr::pack2(acc[6], acc[7]);
  return out;
}

// P:    every rank's partial buffer, global rows, pitch ldp
// R:    [rows][ldr] residual (global rows), or nullptr; bias [N] or nullptr
// Y:    every rank's output buffer, global rows, pitch ldy
// Each thread handles two 16-byte column groups per step (consecutive
// threads on consecutive groups), with all 2 x world loads in flight.
template <typename T>
__global__ void __launch_bounds__(256)
    reduce_broadcast_kernel(RankPtrs P, int world, int rank, int rows_per_rank, int N,
                            long long ldp, const T* __restrict__ bias, const T* __restrict__ R,
                            long long ldr, RankPtrs Y, long long ldy) {
  const int groups = N / 8;  // 8 columns (16 bytes) per group
  const long long total = static_cast<long long>(rows_per_rank) * groups;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  const long long row0 = static_cast<long long>(rank) * rows_per_rank;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += 2 * stride) {
    const long long i2 = i + stride;
    const bool two = i2 < total;
    const int r1 = static_cast<int>(i / groups), c1 = static_cast<int>(i - static_cast<long long>(r1) * groups) * 8;
    const int r2 = two ? static_cast<int>(i2 / groups) : r1;
    const int c2 = two ? static_cast<int>(i2 - static_cast<long long>(r2) * groups) * 8 : c1;
    uint4 pa[8], pb[8];
    rb_load<T>(P, world, (row0 + r1) * ldp + c1, pa);
    if (two) rb_load<T>(P, world, (row0 + r2) * ldp + c2, pb);
    const uint4 oa = rb_finish<T>(pa, world, bias, R, (row0 + r1) * ldr + c1, c1);
    for (int d = 0; d < world; ++d)
      *reinterpret_cast<uint4*>(static_cast<T*>(Y.p[d]) + (row0 + r1) * ldy + c1) = oa;
    if (two) {
      const uint4 ob = rb_finish<T>(pb, world, bias, R, (row0 + r2) * ldr + c2, c2);
      for (int d = 0; d < world; ++d)
        *reinterpret_cast<uint4*>(static_cast<T*>(Y.p[d]) + (row0 + r2) * ldy + c2) = ob;
    }
  }
  __threadfence_system();
}

}  // namespace dx
