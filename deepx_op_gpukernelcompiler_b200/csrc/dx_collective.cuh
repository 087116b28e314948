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
#include "dx_ptx.cuh"

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

// =====================================================================
// Chunked row-parallel reduction that overlaps the GEMMs.
//
// The second GEMM of a row-parallel chain runs in row chunks.  After chunk c
// of every rank's partial is complete, one launch of row_reduce_kernel on a
// side stream (concurrent with the next chunk's GEMMs on the main stream)
//   phase A (reduce-scatter, chunk c): sums this rank's slab of the chunk's
//     rows — rows c0 + rank*rows/world ... — over all ranks' partials (peer
//     loads, rank order, fp32), adds bias and residual once, rounds, and
//     writes the slab into this rank's output and into its own peer-readable
//     slab buffer;
//   phase B (all-gather, an earlier chunk): copies every other rank's slab of
//     that chunk from the peer's slab buffer into this rank's output.
// The output is written only by its own rank, so it can be any device buffer
// the caller owns.  Ranks synchronise through flag words in peer-mapped
// memory, each stamped with the step's epoch (a counter that grows by one per
// step on every rank): PART(c, s) = rank s's partial of chunk c is complete,
// RED(c, s) = rank s's slab of chunk c is in its slab buffer.
// Every wait is bounded (kRowWaitLimitNs); on expiry the kernel reports the
// timeout in the status word and returns.
//
// Where it runs: the tensor-core GEMM kernels keep two spare warps per CTA
// for it (dx_row_reduce_job), so a chunk's reduction runs on the SMs of the
// next GEMM launch while that launch's tensor-core warps compute — a separate
// kernel on another stream could not share those SMs, whose register files
// the GEMM's warps fill.  The reduction of the last chunk, with no GEMM left
// to ride on, runs as the standalone row_reduce_kernel.
// =====================================================================
constexpr int kRowMaxWorld = 8;
constexpr int kRowMaxChunks = 64;
constexpr int kRowThreads = 256;    // standalone kernel: threads per CTA
constexpr int kRowCtasPerSm = 3;    // and resident CTAs per SM (<= 85 registers)
// Flag words per rank: PART[chunk][src], RED[chunk][src], arrival counters.
constexpr int kRowFlagWords = 2 * kRowMaxChunks * kRowMaxWorld + kRowMaxChunks;
constexpr uint64_t kRowWaitLimitNs = 2000ull * 1000ull * 1000ull;  // 2 s

__host__ __device__ constexpr int row_part_flag(int chunk, int src) {
  return chunk * kRowMaxWorld + src;
}
__host__ __device__ constexpr int row_red_flag(int chunk, int src) {
  return (kRowMaxChunks + chunk) * kRowMaxWorld + src;
}
__host__ __device__ constexpr int row_counter(int chunk) {
  return 2 * kRowMaxChunks * kRowMaxWorld + chunk;
}

struct FlagPtrs {
  int* p[kRowMaxWorld];
};

struct RowReduceArgs {
  RankPtrs P;        // partials [M][ldp], every rank
  RankPtrs S;        // slab buffers [2 * M / world][N], every rank
  FlagPtrs F;        // flag words, every rank
  int world, rank, N;
  long long ldp, ldr, ldy;
  long long slab_base;  // first slab-buffer row of this step (epoch parity)
  long long a_row0;     // phase A chunk: first row, rows (0: no phase A), flag index
  int a_rows, a_chunk;
  long long b_row0;     // phase B chunk
  int b_rows, b_chunk;
  const void* bias;     // [N] or nullptr
  const void* R;        // residual [M][ldr] or nullptr
  void* Y;              // this rank's output [M][ldy]
  int epoch;
  // NVLink multicast (NVLS) form, when mc_part != nullptr: the multicast
  // addresses of the partial buffers and of the peer-written output buffers
  // (bound at the same offsets on every rank), and this rank's own view of
  // the latter, pitch ldo.  The slab buffers S are then unused.
  void* mc_part;
  void* mc_out;
  void* out_sym;
  long long ldo;
};

// NVLS: the sum over every rank's copy of 16 bytes (8 fp16/bf16 values) at a
// multicast address, accumulated in fp32 by the switch and rounded to T.
template <typename T>
__device__ __forceinline__ uint4 multimem_ld_reduce_add(const void* mc) {
  uint4 v;
  if constexpr (ElemTraits<T>::kIsBf16)
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(mc)
                 : "memory");
  else
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.f16x2 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(mc)
                 : "memory");
  return v;
}

// NVLS: 16 bytes stored at a multicast address land in every rank's copy.
__device__ __forceinline__ void multimem_st16(void* mc, const uint4& v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc),
               "f"(__uint_as_float(v.x)), "f"(__uint_as_float(v.y)), "f"(__uint_as_float(v.z)),
               "f"(__uint_as_float(v.w))
               : "memory");
}

// Orders this thread's accesses through a multicast address with its
// accesses to the same memory through the ordinary address.
__device__ __forceinline__ void fence_proxy_alias() {
  asm volatile("fence.proxy.alias;" ::: "memory");
}

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Waits until flags[first + s] has reached `epoch` for every s < count other
// than `skip`.  Bounded: false (and the status word set) after the limit.
__device__ __forceinline__ bool row_wait_flags(const int* flags, int first, int count, int skip,
                                               int epoch) {
  const uint64_t t0 = global_timer_ns();
  for (int s = 0; s < count; ++s) {
    if (s == skip) continue;
    while (ld_acquire_sys(flags + first + s) - epoch < 0) {
      if (global_timer_ns() - t0 > kRowWaitLimitNs) {
        report_timeout();
        return false;
      }
      __nanosleep(128);
    }
  }
  return true;
}

// Sums W partials of one 16-byte column group (rank order, fp32), adds bias
// and residual, rounds.  W is the world size when known at compile time, or
// kRowMaxWorld with `world` bounding the ranks used.
template <typename T, int W>
__device__ __forceinline__ uint4 row_finish(const uint4 (&part)[W], int world, const T* bias,
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
  for (int src = 0; src < W; ++src)
    if (W < kRowMaxWorld || src < world) add(part[src]);  // rank order
  if (bias != nullptr) add(__ldg(reinterpret_cast<const uint4*>(bias + c8)));
  if (R != nullptr) add(__ldcs(reinterpret_cast<const uint4*>(R + roff)));
  uint4 out;
  out.x = Tr::pack2(acc[0], acc[1]);
  out.y = Tr::pack2(acc[2], acc[3]);
  out.z = Tr::pack2(acc[4], acc[5]);
  out.w = Tr::pack2(acc[6], acc[7]);
  return out;
}

// The work of one reduction call, spread over `lanes` threads of the grid:
// `gl` is this thread's index among them and `warps` = lanes / 32.  Runs at
// warp granularity (no block-wide barrier), so it serves both the standalone
// kernel and the spare warps of a tensor-core GEMM launch.  The loads are
// latency-bound (a peer's memory is microseconds away), so each thread keeps
// many 16-byte loads in flight: UA column groups x W ranks in phase A, UB
// groups in phase B.  W is the world size when it is 2, 4 or 8 (then the
// loops are fully unrolled), else kRowMaxWorld with a run-time bound.
// Returns early (status word set) if a wait ran out.
template <typename T, int W, int UA, int UB, int UN>
__device__ __forceinline__ void row_reduce_lanes_w(const RowReduceArgs& a, long long gl,
                                                   long long lanes, int warps) {
  const int lane = threadIdx.x & 31;
  const int groups = a.N / 8;  // 16-byte column groups per row
  T* const Y = static_cast<T*>(a.Y);

  if (a.a_rows > 0) {
    // The launch follows the GEMM that wrote chunk a_chunk of the local
    // partial: announce it to every rank.  Every warp stamps the same epoch,
    // so the announcement never waits for one particular warp to run.
    if (lane < a.world) {
      __threadfence_system();
      st_release_sys(a.F.p[lane] + row_part_flag(a.a_chunk, a.rank), a.epoch);
    }
    int ok = 1;
    if (lane == 0)
      ok = row_wait_flags(a.F.p[a.rank], row_part_flag(a.a_chunk, 0), a.world, -1, a.epoch);
    if (!__shfl_sync(0xffffffffu, ok, 0)) return;
    __syncwarp();  // lane 0's acquire orders the whole warp's reads after it

    const int slab = a.a_rows / a.world;
    const long long row0 = a.a_row0 + static_cast<long long>(a.rank) * slab;
    const long long srow0 = a.slab_base + a.a_row0 / a.world;
    const long long total = static_cast<long long>(slab) * groups;
    const T* const bias = static_cast<const T*>(a.bias);
    const T* const R = static_cast<const T*>(a.R);
    T* const Sown = static_cast<T*>(a.S.p[a.rank]);
    if (a.mc_part != nullptr) {
      // The switch sums the ranks' partials; the finished rows go to this
      // rank's output and, by one multicast store, to every rank's buffer.
      const T* const mcp = static_cast<const T*>(a.mc_part);
      T* const mco = static_cast<T*>(a.mc_out);
      for (long long i0 = gl; i0 < total; i0 += UN * lanes) {
        uint4 sum[UN];
#pragma unroll
        for (int u = 0; u < UN; ++u) {
          const long long i = i0 + u * lanes;
          if (i < total) {
            const int r = static_cast<int>(i / groups);
            const int c8 = static_cast<int>(i - static_cast<long long>(r) * groups) * 8;
            sum[u] = multimem_ld_reduce_add<T>(mcp + (row0 + r) * a.ldp + c8);
          }
        }
#pragma unroll
        for (int u = 0; u < UN; ++u) {
          const long long i = i0 + u * lanes;
          if (i < total) {
            const int r = static_cast<int>(i / groups);
            const int c8 = static_cast<int>(i - static_cast<long long>(r) * groups) * 8;
            const uint4 parts[1] = {sum[u]};
            const uint4 o = row_finish<T, 1>(parts, 1, bias, R, (row0 + r) * a.ldr + c8, c8);
            __stcs(reinterpret_cast<uint4*>(Y + (row0 + r) * a.ldy + c8), o);
            multimem_st16(mco + (row0 + r) * a.ldo + c8, o);
          }
        }
      }
      fence_proxy_alias();
    } else
    for (long long i0 = gl; i0 < total; i0 += UA * lanes) {
      uint4 part[UA][W];
#pragma unroll
      for (int u = 0; u < UA; ++u) {
        const long long i = i0 + u * lanes;
        if (i < total) {
          const int r = static_cast<int>(i / groups);
          const int c8 = static_cast<int>(i - static_cast<long long>(r) * groups) * 8;
#pragma unroll
          for (int src = 0; src < W; ++src)
            if (W < kRowMaxWorld || src < a.world)
              part[u][src] = __ldcg(reinterpret_cast<const uint4*>(
                  static_cast<const T*>(a.P.p[src]) + (row0 + r) * a.ldp + c8));
        }
      }
#pragma unroll
      for (int u = 0; u < UA; ++u) {
        const long long i = i0 + u * lanes;
        if (i < total) {
          const int r = static_cast<int>(i / groups);
          const int c8 = static_cast<int>(i - static_cast<long long>(r) * groups) * 8;
          const uint4 o = row_finish<T, W>(part[u], a.world, bias, R, (row0 + r) * a.ldr + c8, c8);
          __stcs(reinterpret_cast<uint4*>(Y + (row0 + r) * a.ldy + c8), o);
          __stcg(reinterpret_cast<uint4*>(Sown + (srow0 + r) * static_cast<long long>(a.N) + c8),
                 o);
        }
      }
    }
    // The last warp to finish announces the slab to every rank.
    __syncwarp();
    if (lane == 0) {
      __threadfence_system();
      int* const ctr = a.F.p[a.rank] + row_counter(a.a_chunk);
      if (atomicAdd(ctr, 1) == warps - 1) {
        atomicExch(ctr, 0);
        __threadfence_system();
        for (int s = 0; s < a.world; ++s)
          st_release_sys(a.F.p[s] + row_red_flag(a.a_chunk, a.rank), a.epoch);
      }
    }
  }

  if (a.b_rows > 0) {
    int ok = 1;
    if (lane == 0)
      ok = row_wait_flags(a.F.p[a.rank], row_red_flag(a.b_chunk, 0), a.world, a.rank, a.epoch);
    if (!__shfl_sync(0xffffffffu, ok, 0)) return;
    __syncwarp();
    const int slab = a.b_rows / a.world;
    const long long srow0 = a.slab_base + a.b_row0 / a.world;
    const long long per_src = static_cast<long long>(slab) * groups;
    const long long total = per_src * (a.world - 1);
    if (a.mc_part != nullptr) {
      // The other ranks' slabs are already in this rank's multicast output
      // buffer (their phase A stored them there): a local copy into Y.
      fence_proxy_alias();
      const T* const osym = static_cast<const T*>(a.out_sym);
      for (long long i0 = gl; i0 < total; i0 += UB * lanes) {
        uint4 v[UB];
        long long dst[UB];
#pragma unroll
        for (int u = 0; u < UB; ++u) {
          const long long i = i0 + u * lanes;
          dst[u] = -1;
          if (i < total) {
            const int k = static_cast<int>(i / per_src);
            const long long j = i - k * per_src;
            const int src = k + (k >= a.rank ? 1 : 0);
            const int r = static_cast<int>(j / groups);
            const int c8 = static_cast<int>(j - static_cast<long long>(r) * groups) * 8;
            const long long row = a.b_row0 + static_cast<long long>(src) * slab + r;
            v[u] = __ldcg(reinterpret_cast<const uint4*>(osym + row * a.ldo + c8));
            dst[u] = row * a.ldy + c8;
          }
        }
#pragma unroll
        for (int u = 0; u < UB; ++u)
          if (dst[u] >= 0) __stcs(reinterpret_cast<uint4*>(Y + dst[u]), v[u]);
      }
      return;
    }
    for (long long i0 = gl; i0 < total; i0 += UB * lanes) {
      uint4 v[UB];
      long long dst[UB];
#pragma unroll
      for (int u = 0; u < UB; ++u) {
        const long long i = i0 + u * lanes;
        dst[u] = -1;
        if (i < total) {
          const int k = static_cast<int>(i / per_src);
          const long long j = i - k * per_src;
          const int src = k + (k >= a.rank ? 1 : 0);
          const int r = static_cast<int>(j / groups);
          const int c8 = static_cast<int>(j - static_cast<long long>(r) * groups) * 8;
          v[u] = __ldcg(reinterpret_cast<const uint4*>(
              static_cast<const T*>(a.S.p[src]) + (srow0 + r) * static_cast<long long>(a.N) + c8));
          dst[u] = (a.b_row0 + static_cast<long long>(src) * slab + r) * a.ldy + c8;
        }
      }
#pragma unroll
      for (int u = 0; u < UB; ++u)
        if (dst[u] >= 0) __stcs(reinterpret_cast<uint4*>(Y + dst[u]), v[u]);
    }
  }
}

// LOADS 16-byte loads in flight per thread in phase A (split over the W
// ranks' partials, or LOADS / 2 multicast reductions), UB in phase B.  A
// peer's memory is several microseconds away under load, so the bandwidth a
// grid reaches is about (threads x bytes in flight) / latency: the GEMM's two
// spare warps per SM keep many loads each (they have the GEMM's register
// budget); the standalone kernel runs more threads with fewer each.
template <typename T, int LOADS, int UB>
__device__ __forceinline__ void row_reduce_lanes(const RowReduceArgs& a, long long gl,
                                                 long long lanes, int warps) {
  constexpr int UN = LOADS / 2;
  switch (a.world) {
    case 2: row_reduce_lanes_w<T, 2, LOADS / 2, UB, UN>(a, gl, lanes, warps); break;
    case 4: row_reduce_lanes_w<T, 4, LOADS / 4, UB, UN>(a, gl, lanes, warps); break;
    case 8: row_reduce_lanes_w<T, 8, LOADS / 8, UB, UN>(a, gl, lanes, warps); break;
    default: row_reduce_lanes_w<T, kRowMaxWorld, LOADS / 8, UB, UN>(a, gl, lanes, warps); break;
  }
}

// Standalone form: the call that ends a step (the last chunk, with nothing
// left to overlap), or a job whose GEMM launch could not carry it.
template <typename T>
__global__ void __launch_bounds__(kRowThreads, kRowCtasPerSm) row_reduce_kernel(const RowReduceArgs a) {
  const long long lanes = static_cast<long long>(gridDim.x) * kRowThreads;
  row_reduce_lanes<T, 12, 8>(a, static_cast<long long>(blockIdx.x) * kRowThreads + threadIdx.x,
                             lanes, static_cast<int>(lanes / 32));
}

}  // namespace dx
