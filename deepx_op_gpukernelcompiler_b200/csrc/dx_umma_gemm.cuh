// dx_umma_gemm.cuh — persistent tcgen05 GEMMs with the fused linear epilogue:
//   Y[M,N] = act(X[M,K] @ W[K,N] + bias[N]) (+ R[M,N]),  fp16/bf16 in and out,
//   fp32 accumulation in TMEM.
//
// This replaces the reference's per-tile K loop + epilogue
// (kernel_triton.py:47-67, kernel_tilelang.py:36-53) with a B200 design.
// Two kernels share one structure:
//
//   umma2_fused_linear_kernel  (main path) — CTA pairs (clusters of 2, one
//     CTA per SM).  A pair owns a 256 x BN output tile: each CTA loads its own
//     128 rows of X and its own BN/2 columns of W, and the leader CTA issues
//     tcgen05.mma.cta_group::2 (M = 256, N = BN, K = 16), which reads A from
//     both CTAs and B from both CTAs and writes each CTA's 128 rows into that
//     CTA's TMEM.  Per SM this halves the W bytes that must be staged in
//     shared memory per MMA compared with a single-CTA 128 x BN tile.
//   umma_fused_linear_kernel   (M < 256) — single CTA, 128 x BN tiles.
//
// Roles inside a CTA (384 threads):
//   warp 0   TMA producer: X tiles [128 x 64] (K-major) and W tiles
//            [64 x 64] boxes (N-major, W exactly as it lies in memory) into
//            a STAGES-deep ring of 128-byte-swizzled buffers;
//   warp 1   TMEM allocator; its lane 0 (in the leader CTA for pairs) issues
//            the MMAs into one of two TMEM accumulators (double buffer);
//   warps 2-9 epilogue: each warp owns the 32 TMEM lanes (= tile rows) it may
//            address (two warps per lane quarter, each taking half of the
//            columns), pulls 32 fp32 columns at a time with tcgen05.ld, adds
//            bias, applies the activation, adds the residual (TMA-loaded into
//            the staging buffer), converts, and TMA-stores.  The output tile
//            crosses HBM exactly once; the next tile's main loop runs in the
//            other accumulator meanwhile;
//   warps 10-11 spare: when the launch carries a row-parallel reduction job
//            (the previous chunk of a row-parallel chain's second GEMM, see
//            dx_collective.cuh), they run it over NVLink while the GEMM
//            computes; otherwise they exit at once.
// Gated form (kGated): Y = act(X Wg + bg) * (X Wu + bu), the first half of a
// gated FFN.  A BN-wide accumulator holds BN/2 gate columns followed by the
// matching BN/2 up columns: the producer fills the B operand's first half
// from Wg and its second half from Wu (for pairs: the leader stages Wg, the
// peer Wu), one MMA covers both, and the epilogue combines column c with
// column c + BN/2 into one output column.  Output tiles are BN/2 wide.
// Tiles are visited M-fastest inside groups of `group_m` m-tiles, so a band
// of X stays in L2 while all of W streams past it; Y and R are streamed with
// an evict-first L2 policy.
// Every mbarrier wait is bounded (dx_ptx.cuh); a timed-out CTA drains its
// copies in flight, frees TMEM and exits with the device status bit set.
#pragma once

#include "dx_collective.cuh"
#include "dx_epilogue.cuh"
#include "dx_ptx.cuh"

namespace dx {

struct UmmaParams {
  int M, N, K;
  int m_tiles, n_tiles, k_blocks, num_tiles;  // tiles of (rows per tile) x BN
  int group_m;                                // m-tiles per raster group
  const void* bias;                           // N elements, or nullptr
  const void* bias2;                          // gated: up-projection bias, or nullptr
  int act;
  int has_residual;
  float alpha;                                // Y = act(alpha * acc + bias) + R
  // Schedule.  The tiles [dp_tiles, num_tiles) that would form a last,
  // partial wave are cut into `splits` pieces along K, one piece per worker
  // (CTA pair or CTA) on workers 0..; each worker processes its piece first,
  // then whole tiles dealt round-robin from [0, dp_tiles).  Pieces leave fp32
  // partial sums in `partials` and finish the tile cooperatively.
  int workers;
  int dp_tiles;
  int splits;
  float* partials;  // [tail tile][split][CTA of the tile][128][BN]
  int* tickets;     // [tail tile][CTA of the tile][kEpiWarps][2]; zero between calls
  // Optional timeline (dx_set_trace_buffer): per CTA kTraceSlots device-time
  // stamps: [0] after set-up, [1 + i] when the epilogue finished work item i
  // (first kTraceSlots - 3 items), [kTraceSlots - 2] when the CTA's spare
  // warps finished a carried reduction job, [kTraceSlots - 1] at exit.
  unsigned long long* trace;
  // A row-parallel reduction job carried by this launch (dx_row_reduce_job):
  // the CTAs' spare warps run it while the other warps compute the GEMM.
  int comm_on;
  RowReduceArgs comm;
};

__device__ __forceinline__ void trace_mark(const UmmaParams& p, int slot) {
  if (p.trace != nullptr && slot < kTraceSlots)
    p.trace[static_cast<size_t>(blockIdx.x) * kTraceSlots + slot] = global_timer_ns();
}

struct WorkItem {
  int tile, kb0, kb1, split;  // split < 0: the whole K range of the tile
};

__device__ __forceinline__ bool umma_item(const UmmaParams& p, int worker, int i, WorkItem& w) {
  // Split pieces (at most one per worker) come first, so their partial-sum
  // traffic and fix-up overlap the whole tiles that follow.
  const int tail_items = (p.num_tiles - p.dp_tiles) * p.splits;
  int j = i;
  if (worker < tail_items) {
    if (i == 0) {
      w.tile = p.dp_tiles + worker / p.splits;
      w.split = worker % p.splits;
      w.kb0 = static_cast<int>((static_cast<long long>(w.split) * p.k_blocks) / p.splits);
      w.kb1 = static_cast<int>((static_cast<long long>(w.split + 1) * p.k_blocks) / p.splits);
      return true;
    }
    j = i - 1;
  }
  const long long idx = static_cast<long long>(worker) + static_cast<long long>(j) * p.workers;
  if (idx >= p.dp_tiles) return false;
  w.tile = static_cast<int>(idx);
  w.kb0 = 0;
  w.kb1 = p.k_blocks;
  w.split = -1;
  return true;
}

__device__ __forceinline__ void umma_tile_coords(const UmmaParams& p, int t, int& mb, int& nb) {
  const int per_group = p.group_m * p.n_tiles;
  const int g = t / per_group;
  const int r = t - g * per_group;
  const int m_first = g * p.group_m;
  const int gm = min(p.group_m, p.m_tiles - m_first);
  mb = m_first + r % gm;
  nb = r / gm;
}

// Epilogue warps: two per TMEM lane quarter, each finishing half of a
// tile's columns, so a tile's epilogue (which overlaps the next tile's main
// loop but is exposed after the last one) takes half as long.
constexpr int kEpiWarps = 8;
constexpr int kEpiHalves = kEpiWarps / 4;
constexpr int kEpiBufBytes = 32 * 32 * 2;  // [32 rows x 32 cols] of 16-bit
// Staging buffers per epilogue warp: a chunk's buffer is reused only after
// the TMA store issued kEpiBufs chunks earlier has read it, so up to
// kEpiBufs - 1 stores stay in flight behind the producer's loads.
constexpr int kEpiBufs = 2;
// Spare warps per CTA (after the epilogue warps) that run a row-parallel
// reduction job when the launch carries one, and otherwise just exit.  With
// them a CTA has 12 warps, three on each of the SM's four sub-partitions,
// whose register files 12 x 168 registers per thread fill (16,128 of 16,384
// each): no other kernel's CTA could be placed beside a GEMM CTA, so work
// that must overlap the GEMM has to live in its launch.
constexpr int kCommWarps = 2;

// The spare warps of every CTA of a GEMM launch run the launch's reduction
// job together (2 warps x grid CTAs).
template <typename T>
__device__ __forceinline__ void comm_warps_run(const UmmaParams& p, int warp, int lane) {
  const int cw = warp - 2 - kEpiWarps;
  const int warps = static_cast<int>(gridDim.x) * kCommWarps;
  const long long gl = (static_cast<long long>(blockIdx.x) * kCommWarps + cw) * 32 + lane;
  row_reduce_lanes<T, 24, 12>(p.comm, gl, static_cast<long long>(warps) * 32, warps);
  if (cw == 0 && lane == 0) trace_mark(p, kTraceSlots - 2);
}

// What one epilogue warp needs to finish accumulators.
template <typename T>
struct EpilogueCtx {
  const CUtensorMap* tmY;
  const CUtensorMap* tmR;
  const T* bias;
  bool bias_vec_ok;
  int M, N, act, has_residual;
  float alpha;
  uint32_t ebuf0;      // this warp's kEpiBufs staging buffers (shared address)
  uint8_t* ebuf_ptr0;  // same, generic pointer
  uint32_t rbar0;      // this warp's kEpiBufs residual-load barriers (8 B apart)
  uint64_t pol_stream; // evict-first policy for Y stores and R loads
};

// Staging-buffer half of a 32-column chunk: waits until the store that last
// used this buffer has read it, and starts the residual tile's TMA load.
template <typename T>
__device__ __forceinline__ void epi_chunk_begin(const EpilogueCtx<T>& c, int n_c, int row_base,
                                                int lane, uint32_t it) {
  const int buf = it % kEpiBufs;
  if (lane == 0) bulk_wait_group_read<kEpiBufs - 1>();
  __syncwarp();
  if (c.has_residual && lane == 0) {
    const uint32_t rbar = c.rbar0 + 8u * buf;
    mbar_arrive_expect_tx(rbar, kEpiBufBytes);
    tma_load_2d_hint(c.tmR, c.ebuf0 + buf * kEpiBufBytes, rbar, n_c, row_base, c.pol_stream);
  }
}

// Finishes a 32-column chunk whose fp32 sums are in v: bias, activation,
// residual, convert, stage (64-byte swizzle) and TMA-store.  Returns false
// if the residual wait gave up.
// Bias of one tile, spread over a warp: lane l holds the 8 values
// bias[n0 + 8l .. n0 + 8l + 8) (zeros past N), loaded before the accumulator
// is ready so its latency is hidden; chunks fetch theirs by warp shuffle.
template <typename T>
__device__ __forceinline__ uint4 epi_load_bias(const EpilogueCtx<T>& c, int n0, int bn, int lane) {
  using Tr = ElemTraits<T>;
  uint4 w = make_uint4(0u, 0u, 0u, 0u);
  const int n = n0 + 8 * lane;
  if (c.bias == nullptr || 8 * lane >= bn || n >= c.N) return w;
  if (c.bias_vec_ok && n + 8 <= c.N) return __ldg(reinterpret_cast<const uint4*>(c.bias + n));
  uint32_t u[4];
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    const float lo = n + 2 * h < c.N ? Tr::to_float(c.bias[n + 2 * h]) : 0.0f;
    const float hi = n + 2 * h + 1 < c.N ? Tr::to_float(c.bias[n + 2 * h + 1]) : 0.0f;
    u[h] = Tr::pack2(lo, hi);
  }
  return make_uint4(u[0], u[1], u[2], u[3]);
}

template <typename T>
__device__ __forceinline__ bool epi_chunk_end(const EpilogueCtx<T>& c, float (&v)[32], int n_c,
                                              int row_base, int lane, uint32_t& it,
                                              volatile int* abort_flag, uint4 bias_reg, int ch) {
  using Tr = ElemTraits<T>;
  const int buf = it % kEpiBufs;
  const uint32_t ebuf = c.ebuf0 + buf * kEpiBufBytes;
  uint8_t* const ebp = c.ebuf_ptr0 + buf * kEpiBufBytes;
  const uint32_t row_off = static_cast<uint32_t>(lane) * 64u;
  const uint32_t row_sw = (static_cast<uint32_t>(lane) >> 1) & 3u;  // 64-byte swizzle phase
  if (c.alpha != 1.0f) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] *= c.alpha;
  }
  if (c.bias != nullptr) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int src = 4 * ch + j;  // lane holding columns n_c + 8j .. n_c + 8j + 8
      const uint32_t wv[4] = {__shfl_sync(0xffffffffu, bias_reg.x, src),
                              __shfl_sync(0xffffffffu, bias_reg.y, src),
                              __shfl_sync(0xffffffffu, bias_reg.z, src),
                              __shfl_sync(0xffffffffu, bias_reg.w, src)};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float2 f = Tr::unpack2(wv[h]);
        v[8 * j + 2 * h] += f.x;
        v[8 * j + 2 * h + 1] += f.y;
      }
    }
  }
  act_apply_all(v, c.act);
  if (c.has_residual) {
    const uint32_t rbar = c.rbar0 + 8u * buf;
    const uint32_t par = (it / kEpiBufs) & 1u;
    if (!mbar_wait(rbar, par, abort_flag)) {
      mbar_wait_drain(rbar, par);  // the load still lands in this buffer
      return false;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 w = *reinterpret_cast<const uint4*>(
          ebp + row_off + ((static_cast<uint32_t>(j) ^ row_sw) << 4));
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
    tma_store_2d_hint(c.tmY, ebuf, n_c, row_base, c.pol_stream);
    bulk_commit_group();
  }
  ++it;
  return true;
}

// Drains this warp's part of one 128 x BN accumulator: TMEM lanes
// [32q, 32q+32), i.e. global rows row0 + 32q + lane, and the 32-column
// chunks [ch0, ch1) of columns n0 .. n0+BN.  `release()` is called (lane 0,
// after the warp's last TMEM read) to hand the accumulator back to the MMA
// issuer.  `it` counts staging-buffer uses.  Returns false if a bounded wait
// gave up.
template <int BN, typename T, typename Release>
__device__ __forceinline__ bool epilogue_tile(const EpilogueCtx<T>& c, uint32_t tmem_acc, int q,
                                              int lane, int row0, int n0, int ch0, int ch1,
                                              uint4 bias_reg, uint32_t& it,
                                              volatile int* abort_flag, Release release) {
  const int row_base = row0 + q * 32;
  const bool rows_live = row_base < c.M;
  const uint32_t lane_addr = tmem_acc + (static_cast<uint32_t>(q * 32) << 16);
  int ce = ch0;  // live chunks are a prefix of the tile's columns
  if (rows_live) {
    const int cols = min(BN, c.N - n0);
    ce = min(ch1, cols > 0 ? (cols + 31) / 32 : 0);
  }
  if (ce <= ch0) {
    tc_fence_before();
    __syncwarp();
    if (lane == 0) release();
    return true;
  }
  // The TMEM load of chunk ch + 1 is in flight while chunk ch is finished.
  uint32_t r[32];
  tmem_ld_32x32b_x32(lane_addr + static_cast<uint32_t>(32 * ch0), r);
#pragma unroll 1
  for (int ch = ch0; ch < ce; ++ch) {
    const int n_c = n0 + 32 * ch;
    epi_chunk_begin(c, n_c, row_base, lane, it);
    tmem_wait_ld();
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
    if (ch + 1 < ce) {
      tmem_ld_32x32b_x32(lane_addr + static_cast<uint32_t>(32 * (ch + 1)), r);
    } else {
      // Accumulator fully read: hand it back to the MMA issuer.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) release();
    }
    if (!epi_chunk_end(c, v, n_c, row_base, lane, it, abort_flag, bias_reg, ch)) {
      if (ch + 1 < ce) tmem_wait_ld();
      return false;
    }
  }
  return true;
}

// Gated form of epilogue_tile: the accumulator holds BN/2 gate columns then
// BN/2 up columns; output column n0 + j = act(gate_j + bg) * (up_j + bu).
// `c` must have no bias, no activation, alpha 1 and no residual (they are
// applied here); the biases arrive spread over the warp as in epi_load_bias.
// The warp handles output chunks [ch0, ch1) (32 columns each).
template <int BN, typename T, typename Release>
__device__ __forceinline__ bool epilogue_tile_gated(const EpilogueCtx<T>& c, uint32_t tmem_acc,
                                                    int q, int lane, int row0, int n0, int ch0,
                                                    int ch1, int act, bool has_bg, bool has_bu,
                                                    uint4 bg_reg, uint4 bu_reg, uint32_t& it,
                                                    volatile int* abort_flag, Release release) {
  using Tr = ElemTraits<T>;
  constexpr int BNO = BN / 2;
  const int row_base = row0 + q * 32;
  const bool rows_live = row_base < c.M;
  const uint32_t lane_addr = tmem_acc + (static_cast<uint32_t>(q * 32) << 16);
  int n_chunks = ch0;
  if (rows_live) {
    const int cols = min(BNO, c.N - n0);
    n_chunks = min(ch1, cols > 0 ? (cols + 31) / 32 : 0);
  }
  if (n_chunks <= ch0) {
    tc_fence_before();
    __syncwarp();
    if (lane == 0) release();
    return true;
  }
  // Both halves of chunk ch + 1 are loading while chunk ch is finished.
  uint32_t rg[32], ru[32];
  tmem_ld_32x32b_x32(lane_addr + static_cast<uint32_t>(32 * ch0), rg);
  tmem_ld_32x32b_x32(lane_addr + static_cast<uint32_t>(BNO + 32 * ch0), ru);
#pragma unroll 1
  for (int ch = ch0; ch < n_chunks; ++ch) {
    const int n_c = n0 + 32 * ch;
    epi_chunk_begin(c, n_c, row_base, lane, it);
    tmem_wait_ld();
    float g[32], u[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      g[j] = __uint_as_float(rg[j]);
      u[j] = __uint_as_float(ru[j]);
    }
    if (ch + 1 < n_chunks) {
      tmem_ld_32x32b_x32(lane_addr + static_cast<uint32_t>(32 * (ch + 1)), rg);
      tmem_ld_32x32b_x32(lane_addr + static_cast<uint32_t>(BNO + 32 * (ch + 1)), ru);
    } else {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) release();
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int src = 4 * ch + j;  // lane holding columns n_c + 8j .. n_c + 8j + 8
      const uint32_t gv[4] = {__shfl_sync(0xffffffffu, bg_reg.x, src),
                              __shfl_sync(0xffffffffu, bg_reg.y, src),
                              __shfl_sync(0xffffffffu, bg_reg.z, src),
                              __shfl_sync(0xffffffffu, bg_reg.w, src)};
      const uint32_t uv[4] = {__shfl_sync(0xffffffffu, bu_reg.x, src),
                              __shfl_sync(0xffffffffu, bu_reg.y, src),
                              __shfl_sync(0xffffffffu, bu_reg.z, src),
                              __shfl_sync(0xffffffffu, bu_reg.w, src)};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float2 fg = Tr::unpack2(gv[h]);
        const float2 fu = Tr::unpack2(uv[h]);
        if (has_bg) {
          g[8 * j + 2 * h] += fg.x;
          g[8 * j + 2 * h + 1] += fg.y;
        }
        if (has_bu) {
          u[8 * j + 2 * h] += fu.x;
          u[8 * j + 2 * h + 1] += fu.y;
        }
      }
    }
    act_apply_all(g, act);
#pragma unroll
    for (int j = 0; j < 32; ++j) g[j] *= u[j];
    if (!epi_chunk_end(c, g, n_c, row_base, lane, it, abort_flag, make_uint4(0u, 0u, 0u, 0u), ch)) {
      if (ch + 1 < n_chunks) tmem_wait_ld();
      return false;
    }
  }
  return true;
}

// Bounded wait until *ctr reaches `target` (other CTAs of this launch add to
// it; all CTAs of the launch are resident).  Returns false on timeout.
__device__ __forceinline__ bool wait_counter(const int* ctr, int target, volatile int* abort_flag) {
  if (*reinterpret_cast<const volatile int*>(ctr) >= target) return true;
  const uint64_t t0 = global_timer_ns();
  uint32_t spins = 0;
  while (*reinterpret_cast<const volatile int*>(ctr) < target) {
    __nanosleep(64);
    if ((++spins & 63u) == 0) {
      if (*abort_flag) return false;
      if (global_timer_ns() - t0 > kWaitLimitNs) {
        *abort_flag = 1;
        report_timeout();
        return false;
      }
    }
  }
  return true;
}

// One K-split piece of a tail tile, for this warp's 32-row slab.  Every
// piece publishes its fp32 partial sums, waits until all `splits` pieces of
// the slab have published, then adds the pieces in split order (a fixed
// order: results do not depend on timing) for its own share of the columns —
// chunks ch with ch % splits == split — and runs the epilogue on them.  The
// last piece to leave resets the slab's two counters (`ctr[0]` arrivals,
// `ctr[1]` departures) to zero.  Returns false if a bounded wait gave up.
// A slab's partials are stored column-quad-major — float offset
// ((col / 4) * 32 + row) * 4 + col % 4 — so each warp-wide float4 access
// covers 512 contiguous bytes.
template <int BN, typename T, typename Release, typename PartBase>
__device__ __forceinline__ bool epilogue_split(const EpilogueCtx<T>& c, uint32_t tmem_acc, int q,
                                               int lane, int row0, int n0, int ch0, int ch1,
                                               uint4 bias_reg, int split, int splits, int* ctr,
                                               PartBase part_base, uint32_t& it,
                                               volatile int* abort_flag, Release release) {
  const size_t slab = static_cast<size_t>(q) * 32 * BN;  // this warp's 32 rows
  // float4 index of (column quad j4, this lane's row) within a slab
  auto quad = [lane](int j4) { return static_cast<size_t>(j4) * 32 + lane; };
  float4* const mine = reinterpret_cast<float4*>(part_base(split) + slab);
  // This warp's chunks [ch0, ch1): written by the same warp of every piece,
  // counted on this warp's own counter pair, then reduced chunk ch by
  // piece ch % splits.
#pragma unroll 1
  for (int ch = ch0; ch < ch1; ++ch) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(tmem_acc + static_cast<uint32_t>(32 * ch) +
                           (static_cast<uint32_t>(q * 32) << 16),
                       r);
    tmem_wait_ld();
    if (ch == ch1 - 1) {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) release();
    }
#pragma unroll
    for (int j = 0; j < 8; ++j)
      mine[quad(8 * ch + j)] =
          make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                      __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
  }
  __threadfence();
  __syncwarp();
  if (lane == 0) atomicAdd(ctr, 1);
  bool ok = true;
  if (lane == 0) ok = wait_counter(ctr, splits, abort_flag);
  ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
  if (!ok) return false;
  __threadfence();
  const int row_base = row0 + q * 32;
  const bool rows_live = row_base < c.M;
#pragma unroll 1
  for (int ch = ch0; ch < ch1; ++ch) {
    if (ch % splits != split) continue;
    const int n_c = n0 + 32 * ch;
    if (!(rows_live && n_c < c.N)) continue;
    epi_chunk_begin(c, n_c, row_base, lane, it);
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = 0.0f;
    // Two splits per step with all 16 loads issued before the adds.
    int sp = 0;
    for (; sp + 1 < splits; sp += 2) {
      const float4* a = reinterpret_cast<const float4*>(part_base(sp) + slab);
      const float4* b = reinterpret_cast<const float4*>(part_base(sp + 1) + slab);
      float4 fa[8], fb[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        fa[j] = __ldcg(a + quad(8 * ch + j));
        fb[j] = __ldcg(b + quad(8 * ch + j));
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v[4 * j] += fa[j].x;
        v[4 * j + 1] += fa[j].y;
        v[4 * j + 2] += fa[j].z;
        v[4 * j + 3] += fa[j].w;
        v[4 * j] += fb[j].x;
        v[4 * j + 1] += fb[j].y;
        v[4 * j + 2] += fb[j].z;
        v[4 * j + 3] += fb[j].w;
      }
    }
    if (sp < splits) {
      const float4* a = reinterpret_cast<const float4*>(part_base(sp) + slab);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 f = __ldcg(a + quad(8 * ch + j));
        v[4 * j] += f.x;
        v[4 * j + 1] += f.y;
        v[4 * j + 2] += f.z;
        v[4 * j + 3] += f.w;
      }
    }
    if (!epi_chunk_end(c, v, n_c, row_base, lane, it, abort_flag, bias_reg, ch)) return false;
  }
  __syncwarp();
  if (lane == 0) {
    const int left = atomicAdd(ctr + 1, 1);
    if (left == splits - 1) {
      // Every piece has seen ctr[0] == splits and finished reading.
      ctr[0] = 0;
      ctr[1] = 0;
    }
  }
  return true;
}

// =====================================================================
// Single-CTA kernel: 128 x BN tiles.
// =====================================================================
template <int BN>
struct UmmaShape {
  static constexpr int BM = 128;
  static constexpr int BK = 64;  // 64 x 16-bit = one 128-byte swizzle row
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BK * BN * 2;
  static constexpr int B_BOX_BYTES = BK * 64 * 2;  // one [64 k x 64 n] TMA box
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (BN == 256) ? 4 : 6;
  static constexpr int TMEM_COLS = 2 * BN;  // two fp32 accumulators
  static constexpr int THREADS = 64 + 32 * (kEpiWarps + kCommWarps);
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + STAGES * A_BYTES;
  static constexpr int OFF_EPI = OFF_B + STAGES * B_BYTES;
  static constexpr int OFF_BAR = OFF_EPI + kEpiWarps * kEpiBufs * kEpiBufBytes;
  // full[STAGES], empty[STAGES], tmem_full[2], tmem_empty[2],
  // residual[kEpiWarps][kEpiBufs], drain
  static constexpr int BAR_FULL = 0;
  static constexpr int BAR_EMPTY = STAGES;
  static constexpr int BAR_TFULL = 2 * STAGES;
  static constexpr int BAR_TEMPTY = 2 * STAGES + 2;
  static constexpr int BAR_RES = 2 * STAGES + 4;
  static constexpr int BAR_DRAIN = BAR_RES + kEpiBufs * kEpiWarps;
  static constexpr int NUM_BARS = BAR_DRAIN + 1;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;  // tmem base, abort flag
  static constexpr int SMEM_BYTES = 1024 + OFF_MISC + 16;
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
  static_assert(BN % 64 == 0 && BN >= 64 && BN <= 256, "UMMA N");
};

template <int BN, typename T, bool kGated = false>
__global__ void __launch_bounds__(UmmaShape<BN>::THREADS, 1)
    umma_fused_linear_kernel(const __grid_constant__ CUtensorMap tmA,
                             const __grid_constant__ CUtensorMap tmB,
                             const __grid_constant__ CUtensorMap tmB2,
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
      mbar_init(bar(S::BAR_TEMPTY + b), kEpiWarps);
    }
    for (int i = 0; i < kEpiBufs * kEpiWarps; ++i) mbar_init(bar(S::BAR_RES + i), 1);
    mbar_init(bar(S::BAR_DRAIN), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (kGated) tma_prefetch_desc(&tmB2);
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
  // Set-up above touched only this CTA's shared memory, TMEM and parameters;
  // global memory may hold the preceding launch's output (inputs, Y, split-K
  // tickets, a carried job's flags), so wait for it before any access.
  grid_dependency_wait();
  grid_launch_dependents();
  if (threadIdx.x == 0) trace_mark(p, 0);

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint64_t pol = make_l2_policy_evict_normal();
      int s = 0;
      uint32_t ph = 0, issued = 0;
      bool ok = true;
      for (int i = 0; ok; ++i) {
        WorkItem w;
        if (!umma_item(p, blockIdx.x, i, w)) break;
        int mb, nb;
        umma_tile_coords(p, w.tile, mb, nb);
        const int m0 = mb * S::BM, n0 = nb * (kGated ? BN / 2 : BN);
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!mbar_wait(bar(S::BAR_EMPTY + s), ph ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t fb = bar(S::BAR_FULL + s);
          mbar_arrive_expect_tx(fb, S::STAGE_BYTES);
          tma_load_2d_hint(&tmA, sA + s * S::A_BYTES, fb, kb * S::BK, m0, pol);
#pragma unroll
          for (int j = 0; j < BN / 64; ++j) {
            if constexpr (kGated) {
              // First half of the boxes from Wg, second half from Wu.
              constexpr int HB = BN / 128;
              tma_load_2d_hint(j < HB ? &tmB : &tmB2, sB + s * S::B_BYTES + j * S::B_BOX_BYTES, fb,
                               n0 + 64 * (j % HB), kb * S::BK, pol);
            } else {
              tma_load_2d_hint(&tmB, sB + s * S::B_BYTES + j * S::B_BOX_BYTES, fb, n0 + 64 * j,
                               kb * S::BK, pol);
            }
          }
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
      for (int i = 0; ok; ++i, ++local) {
        WorkItem w;
        if (!umma_item(p, blockIdx.x, i, w)) break;
        const int b = local & 1;
        const uint32_t use_ph = (static_cast<uint32_t>(local) >> 1) & 1u;
        if (!mbar_wait(bar(S::BAR_TEMPTY + b), use_ph ^ 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(b * BN);
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
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
            umma_f16(d_tmem, ad + 2ull * k, bd + 128ull * k, idesc,
                     (kb != w.kb0 || k != 0) ? 1u : 0u);
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
  } else if (warp < 2 + kEpiWarps) {
    // --------------------------------------------------------- epilogue
    const int e = warp - 2;  // epilogue warp index 0..kEpiWarps-1
    const int q = warp & 3;  // TMEM lane quarter this warp may address
    const int hf = e / 4;    // which share of the tile's columns
    const int ch0 = hf * (BN / 32) / kEpiHalves, ch1 = (hf + 1) * (BN / 32) / kEpiHalves;
    const int gch0 = hf * (BN / 64) / kEpiHalves, gch1 = (hf + 1) * (BN / 64) / kEpiHalves;
    EpilogueCtx<T> c;
    c.tmY = &tmY;
    c.tmR = &tmR;
    c.bias = static_cast<const T*>(p.bias);
    c.bias_vec_ok = c.bias != nullptr && (reinterpret_cast<uintptr_t>(c.bias) & 15u) == 0;
    c.M = p.M;
    c.N = p.N;
    c.act = p.act;
    c.alpha = p.alpha;
    c.has_residual = p.has_residual;
    c.ebuf0 = base + S::OFF_EPI + e * kEpiBufs * kEpiBufBytes;
    c.ebuf_ptr0 = base_ptr + S::OFF_EPI + e * kEpiBufs * kEpiBufBytes;
    c.rbar0 = bar(S::BAR_RES + e * kEpiBufs);
    c.pol_stream = make_l2_policy_evict_first();
    // Gated: biases are added before the activation in epilogue_tile_gated;
    // cg / cu only load them.
    EpilogueCtx<T> cg = c, cu = c;
    if (kGated) {
      cu.bias = static_cast<const T*>(p.bias2);
      cu.bias_vec_ok = cu.bias != nullptr && (reinterpret_cast<uintptr_t>(cu.bias) & 15u) == 0;
      c.bias = nullptr;
      c.act = kActNone;
      c.alpha = 1.0f;
    }
    uint32_t it = 0;
    int local = 0;
    for (int i = 0;; ++i, ++local) {
      WorkItem w;
      if (!umma_item(p, blockIdx.x, i, w)) break;
      const int b = local & 1;
      const uint32_t use_ph = (static_cast<uint32_t>(local) >> 1) & 1u;
      int mb, nb;
      umma_tile_coords(p, w.tile, mb, nb);
      const int n0o = nb * (kGated ? BN / 2 : BN);
      const uint4 bias_reg = epi_load_bias(kGated ? cg : c, n0o, kGated ? BN / 2 : BN, lane);
      const uint4 bias_up = kGated ? epi_load_bias(cu, n0o, BN / 2, lane) : make_uint4(0u, 0u, 0u, 0u);
      if (!mbar_wait(bar(S::BAR_TFULL + b), use_ph, abort_flag)) break;
      tc_fence_after();
      const uint32_t tempty = bar(S::BAR_TEMPTY + b);
      const uint32_t acc = tmem_base + static_cast<uint32_t>(b * BN);
      auto release = [tempty] { mbar_arrive(tempty); };
      bool done;
      if constexpr (kGated) {
        done = epilogue_tile_gated<BN, T>(c, acc, q, lane, mb * S::BM, n0o, gch0, gch1, p.act,
                                          cg.bias != nullptr, cu.bias != nullptr, bias_reg,
                                          bias_up, it, abort_flag, release);
      } else if (w.split < 0) {
        done = epilogue_tile<BN, T>(c, acc, q, lane, mb * S::BM, nb * BN, ch0, ch1, bias_reg, it,
                                    abort_flag, release);
      } else {
        const int tail = w.tile - p.dp_tiles;
        float* const partials = p.partials;
        const int splits = p.splits;
        auto part_base = [partials, tail, splits](int sp) {
          return partials + static_cast<size_t>(tail * splits + sp) * 128 * BN;
        };
        done = epilogue_split<BN, T>(c, acc, q, lane, mb * S::BM, nb * BN, ch0, ch1, bias_reg,
                                     w.split, splits, p.tickets + (tail * kEpiWarps + e) * 2,
                                     part_base, it, abort_flag, release);
      }
      if (!done) break;
      if (e == 0 && lane == 0 && 1 + i < kTraceSlots - 2) trace_mark(p, 1 + i);
    }
    if (lane == 0) bulk_wait_group<0>();
    __syncwarp();
  } else if (p.comm_on) {
    // ------------------------ spare warps: the carried reduction job
    comm_warps_run<T>(p, warp, lane);
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) trace_mark(p, kTraceSlots - 1);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, S::TMEM_COLS);
  }
}

// =====================================================================
// CTA-pair kernel: 256 x BN tiles, tcgen05.mma.cta_group::2.
// =====================================================================
template <int BN>
struct Umma2Shape {
  static constexpr int BM = 128;      // rows per CTA (256 per pair)
  static constexpr int BK = 64;
  static constexpr int BN_CTA = BN / 2;  // W columns staged by each CTA
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BOX_BYTES = BK * 64 * 2;
  static constexpr int B_BYTES = BK * BN_CTA * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;  // per CTA
  static constexpr int STAGES = (BN == 256) ? 6 : 8;
  static constexpr int TMEM_COLS = 2 * BN;  // per CTA: two accumulators of BN fp32 columns
  static constexpr int THREADS = 64 + 32 * (kEpiWarps + kCommWarps);
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + STAGES * A_BYTES;
  static constexpr int OFF_EPI = OFF_B + STAGES * B_BYTES;
  static constexpr int OFF_BAR = OFF_EPI + kEpiWarps * kEpiBufs * kEpiBufBytes;
  static constexpr int BAR_FULL = 0;              // leader only: both CTAs' bytes
  static constexpr int BAR_EMPTY = STAGES;        // both CTAs
  static constexpr int BAR_TFULL = 2 * STAGES;    // both CTAs
  static constexpr int BAR_TEMPTY = 2 * STAGES + 2;  // leader only: 8 warp arrivals
  static constexpr int BAR_RES = 2 * STAGES + 4;
  static constexpr int BAR_DRAIN = BAR_RES + kEpiBufs * kEpiWarps;
  static constexpr int NUM_BARS = BAR_DRAIN + 1;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int SMEM_BYTES = 1024 + OFF_MISC + 16;
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
  static_assert(BN == 128 || BN == 256, "pair tile N");
};

template <int BN, typename T, bool kGated = false>
__global__ void __launch_bounds__(Umma2Shape<BN>::THREADS, 1)
    umma2_fused_linear_kernel(const __grid_constant__ CUtensorMap tmA,
                              const __grid_constant__ CUtensorMap tmB,
                              const __grid_constant__ CUtensorMap tmB2,
                              const __grid_constant__ CUtensorMap tmY,
                              const __grid_constant__ CUtensorMap tmR, const UmmaParams p) {
  using S = Umma2Shape<BN>;
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
  const uint32_t rank = cluster_ctarank();  // 0 = leader of the pair
  const bool leader = rank == 0;
  const int pair = static_cast<int>(blockIdx.x >> 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::STAGES; ++s) {
      mbar_init(bar(S::BAR_FULL + s), 1);
      mbar_init(bar(S::BAR_EMPTY + s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar(S::BAR_TFULL + b), 1);
      mbar_init(bar(S::BAR_TEMPTY + b), 2 * kEpiWarps);
    }
    for (int i = 0; i < kEpiBufs * kEpiWarps; ++i) mbar_init(bar(S::BAR_RES + i), 1);
    mbar_init(bar(S::BAR_DRAIN), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (kGated) tma_prefetch_desc(&tmB2);
    tma_prefetch_desc(&tmY);
    if (p.has_residual) tma_prefetch_desc(&tmR);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_word), S::TMEM_COLS);
    tmem_relinquish_pair();
  }
  // Both CTAs' barriers exist and TMEM is allocated before anyone signals
  // across the pair.
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_word;
  // Set-up above touched only this CTA's shared memory, TMEM and parameters;
  // global memory may hold the preceding launch's output (inputs, Y, split-K
  // tickets, a carried job's flags), so wait for it before any access.
  grid_dependency_wait();
  grid_launch_dependents();
  if (threadIdx.x == 0) trace_mark(p, 0);

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint64_t pol = make_l2_policy_evict_normal();
      int s = 0;
      uint32_t ph = 0, issued = 0;
      bool ok = true;
      for (int i = 0; ok; ++i) {
        WorkItem w;
        if (!umma_item(p, pair, i, w)) break;
        int mb, nb;
        umma_tile_coords(p, w.tile, mb, nb);
        const int m0 = mb * 2 * S::BM + static_cast<int>(rank) * S::BM;
        // Gated: the leader stages Wg's and the peer Wu's BN/2 columns.
        const int n0 = kGated ? nb * S::BN_CTA : nb * BN + static_cast<int>(rank) * S::BN_CTA;
        const CUtensorMap* const mapB = (kGated && rank != 0) ? &tmB2 : &tmB;
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!mbar_wait(bar(S::BAR_EMPTY + s), ph ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          // The leader's full barrier counts both CTAs' bytes.
          if (leader) mbar_arrive_expect_tx(bar(S::BAR_FULL + s), 2 * S::STAGE_BYTES);
          const uint32_t fb = mapa_shared(bar(S::BAR_FULL + s), 0);
          tma_load_2d_pair(&tmA, sA + s * S::A_BYTES, fb, kb * S::BK, m0, pol);
#pragma unroll
          for (int j = 0; j < S::BN_CTA / 64; ++j)
            tma_load_2d_pair(mapB, sB + s * S::B_BYTES + j * S::B_BOX_BYTES, fb, n0 + 64 * j,
                             kb * S::BK, pol);
          ++issued;
          if (++s == S::STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      // The leader observes both CTAs' copies through its full barriers.
      if (leader) {
        const uint32_t n_drain = issued < (uint32_t)S::STAGES ? issued : (uint32_t)S::STAGES;
        for (uint32_t i = issued - n_drain; i < issued; ++i)
          mbar_wait_drain(bar(S::BAR_FULL + (int)(i % S::STAGES)), (i / S::STAGES) & 1u);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ----------------------------------------------- MMA issuer (leader)
    if (leader && lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(Tr::kIsBf16, 256, BN, false, true);
      int s = 0, local = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int i = 0; ok; ++i, ++local) {
        WorkItem w;
        if (!umma_item(p, pair, i, w)) break;
        const int b = local & 1;
        const uint32_t use_ph = (static_cast<uint32_t>(local) >> 1) & 1u;
        if (!mbar_wait(bar(S::BAR_TEMPTY + b), use_ph ^ 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(b * BN);
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!mbar_wait(bar(S::BAR_FULL + s), ph, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = smem_desc_sw128(sA + s * S::A_BYTES, 16, 1024);
          const uint64_t bd = smem_desc_sw128(sB + s * S::B_BYTES, S::B_BOX_BYTES, 1024);
#pragma unroll
          for (int k = 0; k < S::BK / 16; ++k)
            umma_f16_pair(d_tmem, ad + 2ull * k, bd + 128ull * k, idesc,
                          (kb != w.kb0 || k != 0) ? 1u : 0u);
          // Stage s is free in both CTAs once these MMAs have read it.
          umma_commit_pair(mapa_shared(bar(S::BAR_EMPTY + s), 0));
          umma_commit_pair(mapa_shared(bar(S::BAR_EMPTY + s), 1));
          if (++s == S::STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (ok) {
          umma_commit_pair(mapa_shared(bar(S::BAR_TFULL + b), 0));
          umma_commit_pair(mapa_shared(bar(S::BAR_TFULL + b), 1));
        }
      }
      umma_commit_pair(mapa_shared(bar(S::BAR_DRAIN), 0));
      mbar_wait_drain(bar(S::BAR_DRAIN), 0);
    }
    __syncwarp();
  } else if (warp < 2 + kEpiWarps) {
    // --------------------------------------------- epilogue (both CTAs)
    const int e = warp - 2;
    const int q = warp & 3;
    const int hf = e / 4;
    const int ch0 = hf * (BN / 32) / kEpiHalves, ch1 = (hf + 1) * (BN / 32) / kEpiHalves;
    const int gch0 = hf * (BN / 64) / kEpiHalves, gch1 = (hf + 1) * (BN / 64) / kEpiHalves;
    EpilogueCtx<T> c;
    c.tmY = &tmY;
    c.tmR = &tmR;
    c.bias = static_cast<const T*>(p.bias);
    c.bias_vec_ok = c.bias != nullptr && (reinterpret_cast<uintptr_t>(c.bias) & 15u) == 0;
    c.M = p.M;
    c.N = p.N;
    c.act = p.act;
    c.alpha = p.alpha;
    c.has_residual = p.has_residual;
    c.ebuf0 = base + S::OFF_EPI + e * kEpiBufs * kEpiBufBytes;
    c.ebuf_ptr0 = base_ptr + S::OFF_EPI + e * kEpiBufs * kEpiBufBytes;
    c.rbar0 = bar(S::BAR_RES + e * kEpiBufs);
    c.pol_stream = make_l2_policy_evict_first();
    // Gated: biases are added before the activation in epilogue_tile_gated;
    // cg / cu only load them.
    EpilogueCtx<T> cg = c, cu = c;
    if (kGated) {
      cu.bias = static_cast<const T*>(p.bias2);
      cu.bias_vec_ok = cu.bias != nullptr && (reinterpret_cast<uintptr_t>(cu.bias) & 15u) == 0;
      c.bias = nullptr;
      c.act = kActNone;
      c.alpha = 1.0f;
    }
    uint32_t it = 0;
    int local = 0;
    for (int i = 0;; ++i, ++local) {
      WorkItem w;
      if (!umma_item(p, pair, i, w)) break;
      const int b = local & 1;
      const uint32_t use_ph = (static_cast<uint32_t>(local) >> 1) & 1u;
      int mb, nb;
      umma_tile_coords(p, w.tile, mb, nb);
      const int n0o = nb * (kGated ? BN / 2 : BN);
      const uint4 bias_reg = epi_load_bias(kGated ? cg : c, n0o, kGated ? BN / 2 : BN, lane);
      const uint4 bias_up = kGated ? epi_load_bias(cu, n0o, BN / 2, lane) : make_uint4(0u, 0u, 0u, 0u);
      if (!mbar_wait(bar(S::BAR_TFULL + b), use_ph, abort_flag)) break;
      tc_fence_after();
      const uint32_t tempty_leader = mapa_shared(bar(S::BAR_TEMPTY + b), 0);
      const uint32_t acc = tmem_base + static_cast<uint32_t>(b * BN);
      const int row0 = mb * 2 * S::BM + static_cast<int>(rank) * S::BM;
      auto release = [tempty_leader] { mbar_arrive_cluster(tempty_leader); };
      bool done;
      if constexpr (kGated) {
        done = epilogue_tile_gated<BN, T>(c, acc, q, lane, row0, n0o, gch0, gch1, p.act,
                                          cg.bias != nullptr, cu.bias != nullptr, bias_reg,
                                          bias_up, it, abort_flag, release);
      } else if (w.split < 0) {
        done = epilogue_tile<BN, T>(c, acc, q, lane, row0, nb * BN, ch0, ch1, bias_reg, it,
                                    abort_flag, release);
      } else {
        const int tail = w.tile - p.dp_tiles;
        float* const partials = p.partials;
        const int splits = p.splits;
        const int r = static_cast<int>(rank);
        auto part_base = [partials, tail, splits, r](int sp) {
          return partials + (static_cast<size_t>(tail * splits + sp) * 2 + r) * 128 * BN;
        };
        done = epilogue_split<BN, T>(c, acc, q, lane, row0, nb * BN, ch0, ch1, bias_reg, w.split,
                                     splits, p.tickets + ((tail * 2 + r) * kEpiWarps + e) * 2,
                                     part_base, it, abort_flag, release);
      }
      if (!done) break;
      if (e == 0 && lane == 0 && 1 + i < kTraceSlots - 2) trace_mark(p, 1 + i);
    }
    if (lane == 0) bulk_wait_group<0>();
    __syncwarp();
  } else if (p.comm_on) {
    // ------------------------ spare warps: the carried reduction job
    comm_warps_run<T>(p, warp, lane);
  }

  // No CTA of the pair leaves while the other may still signal it.
  tc_fence_before();
  cluster_sync();
  if (threadIdx.x == 0) trace_mark(p, kTraceSlots - 1);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, S::TMEM_COLS);
  }
}

}  // namespace dx
