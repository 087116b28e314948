// dx_decode.cuh — skinny-M (decode) fused linear, HBM-bound:
//   Y[M,N] = act(X[M,K] @ W[K,N] + bias[N]) (+ R),  M <= 64, fp16/bf16.
//
// With M <= 64 every element of W is used at most 64 times, so the kernel's
// job is to stream W from HBM exactly once at full bandwidth.  Design:
//   * swap-AB on the tensor core: D^T[n, m] = sum_k W^T[n, k] X^T[k, m], so
//     the 128-wide UMMA M dimension runs over N (W's contiguous axis, read
//     by TMA straight from its row-major layout as an MN-major operand) and
//     the UMMA N dimension is the padded batch MN = 16/32/64 (X as a K-major
//     operand).  A work unit is 256 columns of W by 64 rows of K: two UMMAs
//     (one per 128-column half) per K=16 step into two TMEM accumulators of
//     128 lanes x MN fp32 columns.  Each W row segment read is 512 B long and
//     each 2 KB X tile serves 32 KB of W.
//   * the (n-tile, k-block) work units are partitioned evenly over the
//     grid, each CTA taking one contiguous range (deep pipeline, one CTA per
//     SM).  The host picks the grid: one CTA per whole tile when there are
//     at least half as many tiles as SMs (no split-K at all), else one CTA
//     per SM, so that every SM streams the same number of bytes and a CTA's
//     range crosses at most a few n-tiles (split-K).
//   * with fewer tiles than SMs/2 (plain form) the CTAs of one tile form a
//     thread-block cluster of C = 2, 4 or 8 (tiles x C <= SMs): each streams
//     1/C of the tile's K range and leaves its fp32 partial in its own shared
//     memory (the idle stage ring); after a cluster barrier CTA c sums column
//     slice c over the cluster's shared memories in rank order and runs the
//     epilogue — no workspace, no counters, no global round trip;
//   * otherwise partial sums of a tile that several CTAs share go to a workspace as
//     fp32; the last CTA to arrive at a tile (atomic counter) sums the
//     others' partials and its own registers in fixed segment order —
//     deterministic, no float atomics — applies bias, activation and
//     residual, stores Y, and resets the counter to 0.  When that tile is
//     the CTA's last work item the partials come in by bulk copies into the
//     then idle W stage ring, all in flight at once.
//   * gated form (p.gated): Y = act(X Wg + bg) * (X Wu + bu).  A work unit
//     covers NH/2 x 128 output columns: its first NH/2 UMMA halves read Wg's
//     columns, the others Wu's same columns; the epilogue combines them.
//     With NH = 4 (M <= 16) each weight's row segment read is 512 B, as in
//     the plain form; NH = 2 (256 B segments) serves M up to 64.
// Bounded waits and exit draining as in dx_umma_gemm.cuh.
#pragma once

#include "dx_epilogue.cuh"
#include "dx_ptx.cuh"

namespace dx {

struct DecodeParams {
  int M, N, K;
  int n_tiles;          // ceil(N / 256); gated: ceil(N / 128)
  int kbt;              // k-blocks (64 deep) per tile
  long long units;      // n_tiles * kbt
  int grid;             // CTAs
  int max_seg;          // partial-sum slots per tile
  long long ldy, ldr;
  const void* bias;     // N elements or nullptr
  const void* residual; // [M, N] (ldr) or nullptr
  void* Y;
  float* partials;      // [n_tiles][max_seg][4][NH][MN][32] fp32 (DecodeShape::QBLK)
  int* tickets;         // [n_tiles][4] (per warp quarter): arrivals | written << 16;
                        // zero between calls
  int act;
  float alpha;          // Y = act(alpha * acc + bias) + R
  int gated;            // Y = act(acc_g + bias) * (acc_u + bias2)
  const void* bias2;    // gated: up-projection bias (N) or nullptr
  int cluster;          // CTAs per tile sharing partials through distributed
                        // shared memory (1: off; grid = n_tiles * cluster)
  // Optional timeline (dx_set_trace_buffer), kTraceSlots stamps per CTA:
  // [0] after set-up, [1] first and [2] last TMA issue, [3] last MMA issue;
  // for the CTA's last work item (warp quarter 0): [4] accumulator ready,
  // [5] accumulator read, [6] arrival counted, [7] own partial published or
  // the others' found written, [8] fix-up sums done, [9] item finished;
  // [10 + i] work item i finished (i < 2), [12] kernel entry, [13] the SM's
  // id, [14] epilogue warps done, [15] exit; cluster form: [6] first cluster
  // barrier passed, [7] slices sent, [8] last cluster barrier passed, [9]
  // columns finished.
  unsigned long long* trace;
};

__device__ __forceinline__ void decode_trace(const DecodeParams& p, int slot) {
  if (p.trace != nullptr)
    p.trace[static_cast<size_t>(blockIdx.x) * kTraceSlots + slot] = global_timer_ns();
}

// NH: 128-column UMMA halves per work unit (2; 4 for the wide gated form).
template <int MN, int NH = 2>
struct DecodeShape {
  static constexpr int NT = 128 * NH;              // W columns staged per work unit
  static constexpr int BK = 64;
  static constexpr int W_BOX_BYTES = 64 * BK * 2;  // [64 k x 64 n]
  static constexpr int HALF_BYTES = 2 * W_BOX_BYTES;
  static constexpr int W_BYTES = NH * HALF_BYTES;  // NT n per stage
  static constexpr int X_BYTES = MN * BK * 2;      // MN rows x 128 B
  static constexpr int STAGE_BYTES = W_BYTES + X_BYTES;
  static constexpr int STAGES = NH == 4 ? 3 : (MN <= 32 ? 6 : 5);
  // two buffers x NH halves x MN fp32 columns, as a power of two >= 32
  static constexpr int ACC_COLS = NH * MN;
  static constexpr int TMEM_COLS = 2 * ACC_COLS < 32 ? 32 : 2 * ACC_COLS;
  static constexpr int THREADS = 192;
  static constexpr int OFF_W = 0;
  static constexpr int OFF_X = OFF_W + STAGES * W_BYTES;
  // Cluster form, 16-row template: a receive area of its own (MN x NT fp32),
  // so a CTA can send its partial's slices as soon as its accumulator is
  // read, whatever its cluster peers' stage rings are still doing.
  static constexpr bool OWN_RECV = MN == 16 && NH == 2;
  static constexpr int OFF_RECV = OFF_X + STAGES * X_BYTES;
  static constexpr int OFF_BAR = OFF_RECV + (OWN_RECV ? MN * NT * 4 : 0);
  static constexpr int BAR_FULL = 0;
  static constexpr int BAR_EMPTY = STAGES;
  static constexpr int BAR_TFULL = 2 * STAGES;
  static constexpr int BAR_TEMPTY = 2 * STAGES + 2;
  static constexpr int BAR_DRAIN = 2 * STAGES + 4;
  static constexpr int BAR_FIX = 2 * STAGES + 5;  // one per epilogue warp quarter
  static constexpr int NUM_BARS = BAR_FIX + 4;
  // Split-K partial sums, per tile: [segment][warp quarter][NH][MN][32 lanes]
  // fp32, so one warp quarter's share of a segment is one contiguous block.
  static constexpr int QBLK = NH * MN * 32;
  // Fix-up staging: once a CTA's last accumulator is ready its W stage ring
  // is idle, and each epilogue warp takes a quarter of it for the other
  // segments' blocks (FIX_CAP blocks per batch of bulk copies).
  static constexpr int FIX_CAP = STAGES * W_BYTES / (4 * QBLK * 4);
  // Cluster form without a receive area of its own: the partial (MN x NT
  // fp32) at the start of the idle ring, the slices received from the
  // cluster (at most MN x NT fp32) after it.
  static constexpr int RECV_OFF = MN * NT * 4;
  static_assert(2 * MN * NT * 4 <= STAGES * W_BYTES, "cluster partial and receive area");
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;  // tmem base, abort flag
  static constexpr int SMEM_BYTES = 1024 + OFF_MISC + 16;
  static_assert(MN == 16 || MN == 32 || MN == 64, "decode batch tile");
  static_assert(NH == 2 || (NH == 4 && MN == 16), "halves per unit");
  static_assert(X_BYTES % 1024 == 0, "X stage alignment");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
  static_assert(FIX_CAP >= 1 && (QBLK * 4) % 16 == 0, "fix-up staging");
};

// CTA whose work range holds unit u (ranges are [g*U/G, (g+1)*U/G)).
__device__ __forceinline__ int decode_cta_of(long long u, long long U, int G) {
  int g = static_cast<int>((u * G) / U);
  while (g + 1 < G && ((static_cast<long long>(g) + 1) * U) / G <= u) ++g;
  return g;
}

// Bounded wait until the high half (partials written) of *ctr reaches
// `target`.  Returns false when the CTA's abort flag is raised or the wait
// exceeded kWaitLimitNs (then it raises both flags itself).
__device__ __forceinline__ bool decode_wait_written(const int* ctr, int target,
                                                    volatile int* abort_flag) {
  const uint64_t t0 = global_timer_ns();
  uint32_t spins = 0;
  while ((*reinterpret_cast<const volatile int*>(ctr) >> 16) < target) {
    __nanosleep(32);
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

// Cluster form (plain decode: NH = 2, NT = 256 columns per tile, C = 2, 4
// or 8 CTAs per cluster): rank c of the cluster finishes columns
// c * NT/C .. (c+1) * NT/C - 1 of the tile; log2 of that slice width.
__device__ __forceinline__ int decode_cluster_slice_log2(int C) { return 8 - (31 - __clz(C)); }

// Cluster form: the bias of the column this epilogue thread finishes (each
// thread keeps one column: NT/C divides the 128 epilogue threads).
template <int MN, typename T, int NH>
__device__ __forceinline__ float decode_cluster_bias(const DecodeParams& p) {
  using S = DecodeShape<MN, NH>;
  using Tr = ElemTraits<T>;
  const int lg = decode_cluster_slice_log2(p.cluster);
  const int col = (static_cast<int>(cluster_ctarank()) << lg) +
                  ((static_cast<int>(threadIdx.x) - 64) & ((1 << lg) - 1));
  const int n = static_cast<int>(blockIdx.x) / p.cluster * S::NT + col;
  const T* const bias = static_cast<const T*>(p.bias);
  return (bias != nullptr && n < p.N) ? Tr::to_float(bias[n]) : 0.0f;
}

// Cluster form, sending: each epilogue thread (64..191) takes column
// quarter*32 + lane of both halves and sends its rows to the CTA that
// finishes that column, into that CTA's receive area [source rank][row]
// [column of the slice] (a warp's 32 columns are one 128-byte run there).
// Remote stores need no round trip; the next cluster barrier makes them
// visible.  The 16-row template sends from registers as soon as its
// accumulator is read (decode_cluster_send); the others leave the partial
// in their idle stage ring at `part_s` ([warp quarter][half][row][32 lanes]
// fp32) and send it after a cluster barrier that says every ring is idle
// (decode_cluster_push), into the ring behind the partial.
// Send rows 0..M-1 of column h * 128 + ql (v[m]) to the CTA finishing it,
// into its receive area at `recv_s` (the same offset in every CTA).
template <int MN>
__device__ __forceinline__ void decode_cluster_send(const DecodeParams& p, uint32_t recv_s,
                                                    int h, int ql, const float (&v)[MN]) {
  const int lg = decode_cluster_slice_log2(p.cluster);
  const int ncols = 1 << lg;
  const int col = h * 128 + ql;
  const uint32_t dst = mapa_shared(
      recv_s + static_cast<uint32_t>(
                   (static_cast<int>(cluster_ctarank()) * p.M * ncols + (col & (ncols - 1))) * 4),
      static_cast<uint32_t>(col >> lg));
#pragma unroll
  for (int m = 0; m < MN; ++m)
    if (m < p.M) st_shared_cluster_f32(dst + static_cast<uint32_t>(m * ncols * 4), v[m]);
}

template <int MN, int NH>
__device__ __forceinline__ void decode_cluster_push(const DecodeParams& p, uint32_t part_s,
                                                    uint32_t recv_s) {
  const int ql = static_cast<int>(threadIdx.x) - 64;  // quarter * 32 + lane
  const float* const part = reinterpret_cast<const float*>(__cvta_shared_to_generic(part_s));
#pragma unroll
  for (int h = 0; h < NH; ++h) {
    const float* const src = part + (((ql >> 5) * NH + h) * MN) * 32 + (ql & 31);
    float v[MN];
#pragma unroll
    for (int m = 0; m < MN; ++m) v[m] = m < p.M ? src[m * 32] : 0.0f;
    decode_cluster_send<MN>(p, recv_s, h, ql, v);
  }
}

// Cluster form, step 2 (after the next cluster barrier): this CTA's column
// slice, summed over the C source ranks in rank order from its own receive
// area (deterministic), then bias, activation and residual.  Thread ql takes
// column ql % (NT/C) and every (128 / (NT/C))-th row from ql / (NT/C).
template <int MN, typename T, int NH>
__device__ __forceinline__ void decode_cluster_finish(const DecodeParams& p, uint32_t recv_s,
                                                      float bias) {
  using S = DecodeShape<MN, NH>;
  using Tr = ElemTraits<T>;
  constexpr int kRows = 4;  // rows whose loads are issued together
  const int C = p.cluster;
  const int lg = decode_cluster_slice_log2(C);
  const int ncols = 1 << lg;
  const int tpc = 128 >> lg;  // threads per column
  const int M = p.M;
  const int ql = static_cast<int>(threadIdx.x) - 64;
  const int c = ql & (ncols - 1);
  const int n = static_cast<int>(blockIdx.x) / C * S::NT +
                (static_cast<int>(cluster_ctarank()) << lg) + c;
  if (n >= p.N) return;
  const float* const recv = reinterpret_cast<const float*>(__cvta_shared_to_generic(recv_s));
  const T* const res = static_cast<const T*>(p.residual);
  T* const Y = static_cast<T*>(p.Y);
  for (int m0 = ql >> lg; m0 < M; m0 += kRows * tpc) {
    float sum[kRows], rv[kRows];
#pragma unroll
    for (int i = 0; i < kRows; ++i) {
      const int m = m0 + i * tpc;
      float s = 0.0f;
      rv[i] = 0.0f;
      if (m < M) {
#pragma unroll
        for (int r = 0; r < 8; ++r)
          if (r < C) s += recv[(r * M + m) * ncols + c];
        if (res != nullptr) rv[i] = Tr::to_float(res[m * p.ldr + n]);
      }
      sum[i] = s;
    }
#pragma unroll
    for (int i = 0; i < kRows; ++i) {
      const int m = m0 + i * tpc;
      if (m >= M) break;
      float y = fmaf(p.alpha, sum[i], bias);
      y = act_apply<true>(y, p.act);
      if (res != nullptr) y += rv[i];
      Y[m * p.ldy + n] = Tr::from_float(y);
    }
  }
}

template <int MN, typename T, int NH = 2>
__global__ void __launch_bounds__(DecodeShape<MN, NH>::THREADS, 1)
    decode_fused_linear_kernel(const __grid_constant__ CUtensorMap tmW,
                               const __grid_constant__ CUtensorMap tmW2,
                               const __grid_constant__ CUtensorMap tmX, const DecodeParams p) {
  using S = DecodeShape<MN, NH>;
  using Tr = ElemTraits<T>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t base = (raw_u32 + 1023u) & ~1023u;
  uint8_t* const base_ptr = smem_raw + (base - raw_u32);

  const uint32_t sW = base + S::OFF_W;
  const uint32_t sX = base + S::OFF_X;
  const uint32_t bars = base + S::OFF_BAR;
  uint32_t* const tmem_word = reinterpret_cast<uint32_t*>(base_ptr + S::OFF_MISC);
  volatile int* const abort_flag = reinterpret_cast<volatile int*>(base_ptr + S::OFF_MISC + 4);
  auto bar = [bars](int i) { return bars + 8u * static_cast<uint32_t>(i); };

  if (threadIdx.x == 0) decode_trace(p, 12);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = blockIdx.x;
  const long long U = p.units;
  const long long u_begin = (static_cast<long long>(g) * U) / p.grid;
  const long long u_end = (static_cast<long long>(g + 1) * U) / p.grid;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::STAGES; ++s) {
      mbar_init(bar(S::BAR_FULL + s), 1);
      mbar_init(bar(S::BAR_EMPTY + s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar(S::BAR_TFULL + b), 1);
      mbar_init(bar(S::BAR_TEMPTY + b), 4);
    }
    mbar_init(bar(S::BAR_DRAIN), 1);
    for (int w = 0; w < 4; ++w) mbar_init(bar(S::BAR_FIX + w), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmW);
    if (p.gated) tma_prefetch_desc(&tmW2);
    tma_prefetch_desc(&tmX);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_word), S::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_word;
  // Cluster form: the first phase of the cluster barrier, waited for before
  // any CTA writes into another's shared memory (every CTA has started).
  if (p.cluster > 1) cluster_arrive_relaxed();
  bool cluster_waited = false;  // this thread has waited for that phase
  float cluster_bias = 0.0f;    // the bias of the column it finishes
  // Global memory only after the preceding launch has completed (see
  // grid_dependency_wait); the set-up above overlaps its tail.
  grid_dependency_wait();
  grid_launch_dependents();
  if (threadIdx.x == 0) {
    decode_trace(p, 0);
    if (p.trace != nullptr) {
      uint32_t smid;
      asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
      p.trace[static_cast<size_t>(blockIdx.x) * kTraceSlots + 13] = smid;
    }
  }

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      // W is read exactly once: evict-first, so it does not push the split-K
      // partials (read back by the tile's last CTA) out of L2.
      const uint64_t pol_w = make_l2_policy_evict_first();
      int s = 0;
      uint32_t ph = 0, issued = 0;
      bool ok = true;
      for (long long u = u_begin; ok && u < u_end;) {
        const int t = static_cast<int>(u / p.kbt);
        const int kb0 = static_cast<int>(u - static_cast<long long>(t) * p.kbt);
        const int kb1 = static_cast<int>(p.kbt < kb0 + (u_end - u) ? (long long)p.kbt : kb0 + (u_end - u));
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(bar(S::BAR_EMPTY + s), ph ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t fb = bar(S::BAR_FULL + s);
          mbar_arrive_expect_tx(fb, S::STAGE_BYTES);
#pragma unroll
          for (int j = 0; j < 2 * NH; ++j) {
            // Gated: halves 0 .. NH/2-1 from Wg, the rest from Wu, at the
            // unit's NH/2 x 128 output columns.
            const int h = j >> 1;
            const CUtensorMap* const mw = (p.gated && h >= NH / 2) ? &tmW2 : &tmW;
            const int col = p.gated ? t * (S::NT / 2) + (h % (NH / 2)) * 128 + 64 * (j & 1)
                                    : t * S::NT + 64 * j;
            tma_load_2d_hint(mw, sW + s * S::W_BYTES + j * S::W_BOX_BYTES, fb, col, kb * S::BK,
                             pol_w);
          }
          tma_load_2d(&tmX, sX + s * S::X_BYTES, fb, kb * S::BK, 0);
          if (issued == 0) decode_trace(p, 1);
          ++issued;
          if (++s == S::STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        u += kb1 - kb0;
      }
      decode_trace(p, 2);
      const uint32_t n_drain = issued < (uint32_t)S::STAGES ? issued : (uint32_t)S::STAGES;
      for (uint32_t i = issued - n_drain; i < issued; ++i)
        mbar_wait_drain(bar(S::BAR_FULL + (int)(i % S::STAGES)), (i / S::STAGES) & 1u);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(Tr::kIsBf16, 128, MN, true, false);
      int s = 0, local = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (long long u = u_begin; ok && u < u_end; ++local) {
        const int t = static_cast<int>(u / p.kbt);
        const int kb0 = static_cast<int>(u - static_cast<long long>(t) * p.kbt);
        const int kb1 = static_cast<int>(p.kbt < kb0 + (u_end - u) ? (long long)p.kbt : kb0 + (u_end - u));
        u += kb1 - kb0;
        const int b = local & 1;
        const uint32_t use_ph = (static_cast<uint32_t>(local) >> 1) & 1u;
        if (!mbar_wait(bar(S::BAR_TEMPTY + b), use_ph ^ 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(b * S::ACC_COLS);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(bar(S::BAR_FULL + s), ph, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // X tile: K-major rows of 128 B, 8-row groups 1024 B apart.
          const uint64_t bd = smem_desc_sw128(sX + s * S::X_BYTES, 16, 1024);
#pragma unroll
          for (int h = 0; h < NH; ++h) {
            // W^T half: MN-major (n contiguous), two 64-wide n groups one box
            // apart, 8-row k groups 1024 B apart; +2048 B per K=16 step.
            const uint64_t ad =
                smem_desc_sw128(sW + s * S::W_BYTES + h * S::HALF_BYTES, S::W_BOX_BYTES, 1024);
#pragma unroll
            for (int k = 0; k < S::BK / 16; ++k)
              umma_f16(d_tmem + static_cast<uint32_t>(h * MN), ad + 128ull * k, bd + 2ull * k,
                       idesc, (kb != kb0 || k != 0) ? 1u : 0u);
          }
          umma_commit(bar(S::BAR_EMPTY + s));
          if (++s == S::STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (ok) umma_commit(bar(S::BAR_TFULL + b));
      }
      decode_trace(p, 3);
      umma_commit(bar(S::BAR_DRAIN));
      mbar_wait_drain(bar(S::BAR_DRAIN), 0);
    }
    __syncwarp();
  } else {
    // --------------------------------------------------------- epilogue
    // Cluster form: the bias this thread needs for its finishing column,
    // loaded now -- at the end, behind the cluster's last weight loads in the
    // HBM queues, a single load takes microseconds.
    if constexpr (NH == 2)
      if (p.cluster > 1) cluster_bias = decode_cluster_bias<MN, T, NH>(p);
    const int q = warp & 3;
    const int n_local = q * 32 + lane;
    const T* const bias = static_cast<const T*>(p.bias);
    const T* const bias2 = static_cast<const T*>(p.bias2);
    const T* const res = static_cast<const T*>(p.residual);
    T* const Y = static_cast<T*>(p.Y);
    const int M = p.M;
    int local = 0;
    for (long long u = u_begin; u < u_end; ++local) {
      const int t = static_cast<int>(u / p.kbt);
      const int kb0 = static_cast<int>(u - static_cast<long long>(t) * p.kbt);
      const int kb1 = static_cast<int>(p.kbt < kb0 + (u_end - u) ? (long long)p.kbt : kb0 + (u_end - u));
      u += kb1 - kb0;
      const int b = local & 1;
      const uint32_t use_ph = (static_cast<uint32_t>(local) >> 1) & 1u;
      // The item's bias, loaded while its accumulator is still being built
      // (gated: bv[hp] gate and bv[hp + NH/2] up bias of output column
      // t * NT/2 + hp * 128 + n_local).
      float bv[NH];
      if (p.gated) {
#pragma unroll
        for (int hp = 0; hp < NH / 2; ++hp) {
          const int n = t * (S::NT / 2) + hp * 128 + n_local;
          bv[hp] = (bias != nullptr && n < p.N) ? Tr::to_float(bias[n]) : 0.0f;
          bv[hp + NH / 2] = (bias2 != nullptr && n < p.N) ? Tr::to_float(bias2[n]) : 0.0f;
        }
      } else {
#pragma unroll
        for (int h = 0; h < NH; ++h) {
          const int n = t * S::NT + h * 128 + n_local;
          bv[h] = (bias != nullptr && n < p.N) ? Tr::to_float(bias[n]) : 0.0f;
        }
      }
      if (!mbar_wait(bar(S::BAR_TFULL + b), use_ph, abort_flag)) break;
      tc_fence_after();
      const bool tr = q == 0 && lane == 0;
      if (tr) decode_trace(p, 4);
      float acc[NH][MN];
#pragma unroll
      for (int h = 0; h < NH; ++h) {
        const uint32_t taddr = tmem_base + static_cast<uint32_t>(b * S::ACC_COLS + h * MN) +
                               (static_cast<uint32_t>(q * 32) << 16);
        if constexpr (MN == 16) {
          uint32_t r[16];
          tmem_ld_32x32b_x16(taddr, r);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) acc[h][j] = __uint_as_float(r[j]);
        } else {
#pragma unroll
          for (int c = 0; c < MN / 32; ++c) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(taddr + 32u * c, r);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; ++j) acc[h][32 * c + j] = __uint_as_float(r[j]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(S::BAR_TEMPTY + b));
      if (tr) decode_trace(p, 5);

      if (!(kb0 == 0 && kb1 == p.kbt) && p.cluster > 1) {
        // Cluster form: this CTA's one work item.
        if constexpr (S::OWN_RECV) {
          // Straight from registers to the finishing CTAs' receive areas,
          // once every CTA of the cluster has started.
          cluster_wait();
          cluster_waited = true;
#pragma unroll
          for (int h = 0; h < NH; ++h) decode_cluster_send<MN>(p, base + S::OFF_RECV, h, n_local, acc[h]);
          if (tr) decode_trace(p, 7);
        } else {
          // The stage ring is idle (every MMA that read it has completed):
          // the partial goes there, sent after the cluster barrier below.
          fence_proxy_async_smem();
          float* const part = reinterpret_cast<float*>(base_ptr + S::OFF_W);
#pragma unroll
          for (int h = 0; h < NH; ++h)
#pragma unroll
            for (int m = 0; m < MN; ++m)
              if (m < M) part[((q * NH + h) * MN + m) * 32 + lane] = acc[h][m];
        }
        continue;
      }
      if (!(kb0 == 0 && kb1 == p.kbt)) {
        // Tile shared with other CTAs.  One counter word per (tile, warp
        // quarter): arrivals in the low 16 bits, partials written in the high
        // 16 bits.  Each CTA arrives first; the last to arrive keeps its sums
        // in registers, every other one publishes its partial (this warp's
        // [NH][MN][32] block of the segment, lanes contiguous in n) and then
        // counts it written.  Each warp finishes its own NH x 32 columns, so
        // no cross-warp barrier can be left waiting on an exit.
        const int first = decode_cta_of(static_cast<long long>(t) * p.kbt, U, p.grid);
        const int last = decode_cta_of(static_cast<long long>(t + 1) * p.kbt - 1, U, p.grid);
        const int nseg = last - first + 1;
        const int own = g - first;
        float* const part_t = p.partials + static_cast<size_t>(t) * p.max_seg * MN * S::NT;
        // Offset of (half h, row m) in this warp's block of a segment.
        auto pidx = [q, lane](int h, int m) { return (q * NH + h) * (MN * 32) + m * 32 + lane; };
        int* const ctr = p.tickets + t * 4 + q;
        int old = 0;
        if (lane == 0) old = atomicAdd(ctr, 1);
        old = __shfl_sync(0xffffffffu, old, 0);
        if (tr) decode_trace(p, 6);
        if ((old & 0xffff) != nseg - 1) {
          float* const mine = part_t + static_cast<size_t>(own) * MN * S::NT;
#pragma unroll
          for (int h = 0; h < NH; ++h)
#pragma unroll
            for (int m = 0; m < MN; ++m)
              if (m < M) mine[pidx(h, m)] = acc[h][m];
          fence_proxy_async_global();  // the last CTA may read it with bulk copies
          __threadfence();
          __syncwarp();
          if (lane == 0) atomicAdd(ctr, 1 << 16);
          if (tr) {
            decode_trace(p, 7);
            decode_trace(p, 9);
            if (local < 2) decode_trace(p, 10 + local);
          }
          continue;
        }
        // Last to arrive: the other nseg - 1 CTAs have arrived; wait (bounded)
        // until their partials are written — usually long done.
        int ok = 1;
        if (lane == 0 && (old >> 16) != nseg - 1)
          ok = decode_wait_written(ctr, nseg - 1, abort_flag) ? 1 : 0;
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        __threadfence();
        if (tr) decode_trace(p, 7);
        // Fixed summation order over segments (0 + s_0 + s_1 + ...): bitwise
        // identical results whichever CTA finishes last.
        if constexpr (MN == 64) {
          // Registers cannot hold a second [NH][64] array: this CTA's segment
          // goes through memory like the others, one half-tile at a time.
          float* const mine = part_t + static_cast<size_t>(own) * MN * S::NT;
#pragma unroll
          for (int h = 0; h < NH; ++h)
#pragma unroll
            for (int m = 0; m < MN; ++m) {
              if (m < M) mine[pidx(h, m)] = acc[h][m];
              acc[h][m] = 0.0f;
            }
          for (int sg = 0; sg < nseg; ++sg) {
            const float* src = part_t + static_cast<size_t>(sg) * MN * S::NT;
#pragma unroll
            for (int h = 0; h < NH; ++h) {
              float fv[MN];
#pragma unroll
              for (int m = 0; m < MN; ++m)
                fv[m] = m < M ? __ldcg(src + pidx(h, m)) : 0.0f;
#pragma unroll
              for (int m = 0; m < MN; ++m) acc[h][m] += fv[m];
            }
          }
        } else if (u == u_end) {
          // The CTA's last item: every MMA that read its W stage ring has
          // completed, so this warp's quarter of the ring stages the other
          // segments' blocks (first M rows of each half), FIX_CAP segments per
          // batch of bulk copies: one L2 round trip per batch.  The sum order
          // is the register path's, so the bits do not depend on the path.
          const int n_other = nseg - 1;
          const uint32_t sbuf = sW + static_cast<uint32_t>(q * S::FIX_CAP * S::QBLK * 4);
          const float* const lbuf =
              reinterpret_cast<const float*>(base_ptr + S::OFF_W) + q * S::FIX_CAP * S::QBLK;
          const uint32_t fbar = bar(S::BAR_FIX + q);
          const uint32_t rows_bytes = static_cast<uint32_t>(M) * 32u * 4u;
          float sum[NH][MN];
#pragma unroll
          for (int h = 0; h < NH; ++h)
#pragma unroll
            for (int m = 0; m < MN; ++m) sum[h][m] = 0.0f;
          uint32_t fph = 0;
          bool fok = true;
          fence_proxy_async_global();
          for (int o0 = 0; o0 < n_other; o0 += S::FIX_CAP) {
            const int nb = n_other - o0 < S::FIX_CAP ? n_other - o0 : S::FIX_CAP;
            if (lane == 0) mbar_arrive_expect_tx(fbar, static_cast<uint32_t>(nb * NH) * rows_bytes);
            __syncwarp();
            for (int j = lane; j < nb * NH; j += 32) {
              const int i = j / NH, h = j - (j / NH) * NH;
              const int o = o0 + i;
              const int sg = o < own ? o : o + 1;
              bulk_load_g2s(sbuf + static_cast<uint32_t>((i * S::QBLK + h * MN * 32) * 4),
                            part_t + static_cast<size_t>(sg) * MN * S::NT + (q * NH + h) * (MN * 32),
                            rows_bytes, fbar);
            }
            if (!__all_sync(0xffffffffu, mbar_wait(fbar, fph, abort_flag))) {
              if (lane == 0) mbar_wait_drain(fbar, fph);  // copies in flight land first
              fok = false;
              break;
            }
            for (int i = 0; i < nb; ++i) {
              if (o0 + i == own) {  // segment `own` precedes this one (segment own + 1)
#pragma unroll
                for (int h = 0; h < NH; ++h)
#pragma unroll
                  for (int m = 0; m < MN; ++m) sum[h][m] += acc[h][m];
              }
#pragma unroll
              for (int h = 0; h < NH; ++h)
#pragma unroll
                for (int m = 0; m < MN; ++m)
                  if (m < M) sum[h][m] += lbuf[i * S::QBLK + (h * MN + m) * 32 + lane];
            }
            // All lanes have read the batch before the next one overwrites it.
            __syncwarp();
            fence_proxy_async_smem();
            fph ^= 1u;
          }
          if (!fok) break;
          if (own == n_other) {  // this CTA's segment is the tile's last
#pragma unroll
            for (int h = 0; h < NH; ++h)
#pragma unroll
              for (int m = 0; m < MN; ++m) sum[h][m] += acc[h][m];
          }
#pragma unroll
          for (int h = 0; h < NH; ++h)
#pragma unroll
            for (int m = 0; m < MN; ++m) acc[h][m] = sum[h][m];
        } else {
          // This CTA's segment comes from registers.  The loads of SB other
          // segments are issued before any of them is added, so a tile split
          // over many CTAs costs few memory round trips.  Each pass loads LH
          // halves of SB segments.
          constexpr int LH = NH < 64 / MN ? NH : 64 / MN;
          constexpr int SB = 96 / (LH * MN) > 1 ? 96 / (LH * MN) : 1;
          const int n_other = nseg - 1;
          float sum[NH][MN];
#pragma unroll
          for (int h = 0; h < NH; ++h)
#pragma unroll
            for (int m = 0; m < MN; ++m) sum[h][m] = 0.0f;
          for (int o0 = 0; o0 < n_other; o0 += SB) {
#pragma unroll
            for (int h0 = 0; h0 < NH; h0 += LH) {
              float f[SB][LH][MN];
#pragma unroll
              for (int sb = 0; sb < SB; ++sb) {
                const int o = o0 + sb;
                const int sg = o < own ? o : o + 1;
                const float* src = part_t + static_cast<size_t>(sg) * MN * S::NT;
#pragma unroll
                for (int hh = 0; hh < LH; ++hh)
#pragma unroll
                  for (int m = 0; m < MN; ++m)
                    f[sb][hh][m] = (o < n_other && m < M)
                                       ? __ldcg(src + pidx(h0 + hh, m))
                                       : 0.0f;
              }
#pragma unroll
              for (int sb = 0; sb < SB; ++sb) {
                const int o = o0 + sb;
                if (o < n_other) {
                  if (o == own) {  // segment `own` precedes this one (segment own + 1)
#pragma unroll
                    for (int hh = 0; hh < LH; ++hh)
#pragma unroll
                      for (int m = 0; m < MN; ++m) sum[h0 + hh][m] += acc[h0 + hh][m];
                  }
#pragma unroll
                  for (int hh = 0; hh < LH; ++hh)
#pragma unroll
                    for (int m = 0; m < MN; ++m) sum[h0 + hh][m] += f[sb][hh][m];
                }
              }
            }
          }
          if (own == n_other) {  // this CTA's segment is the tile's last
#pragma unroll
            for (int h = 0; h < NH; ++h)
#pragma unroll
              for (int m = 0; m < MN; ++m) sum[h][m] += acc[h][m];
          }
#pragma unroll
          for (int h = 0; h < NH; ++h)
#pragma unroll
            for (int m = 0; m < MN; ++m) acc[h][m] = sum[h][m];
        }
        if (lane == 0) *ctr = 0;  // every CTA of the tile has arrived and written
        if (tr) decode_trace(p, 8);
      }
      // Rows in groups of 4: the activation runs over a group's values at
      // once (act_apply_all), so their math chains overlap.
#pragma unroll
      for (int m0 = 0; m0 < MN; m0 += 4) {
        if (m0 >= M) continue;
        if (p.gated) {
          float gv[NH / 2 * 4];
#pragma unroll
          for (int hp = 0; hp < NH / 2; ++hp)
#pragma unroll
            for (int i = 0; i < 4; ++i) gv[hp * 4 + i] = acc[hp][m0 + i] + bv[hp];
          act_apply_all(gv, p.act);
#pragma unroll
          for (int hp = 0; hp < NH / 2; ++hp) {
            const int n = t * (S::NT / 2) + hp * 128 + n_local;
            if (n < p.N) {
#pragma unroll
              for (int i = 0; i < 4; ++i)
                if (m0 + i < M)
                  Y[(m0 + i) * p.ldy + n] = Tr::from_float(
                      gv[hp * 4 + i] * (acc[hp + NH / 2][m0 + i] + bv[hp + NH / 2]));
            }
          }
        } else {
          float yv[NH * 4];
#pragma unroll
          for (int h = 0; h < NH; ++h)
#pragma unroll
            for (int i = 0; i < 4; ++i) yv[h * 4 + i] = fmaf(p.alpha, acc[h][m0 + i], bv[h]);
          act_apply_all(yv, p.act);
#pragma unroll
          for (int h = 0; h < NH; ++h) {
            const int n = t * S::NT + h * 128 + n_local;
            if (n < p.N) {
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int m = m0 + i;
                if (m < M) {
                  float y = yv[h * 4 + i];
                  if (res != nullptr) y += Tr::to_float(res[m * p.ldr + n]);
                  Y[m * p.ldy + n] = Tr::from_float(y);
                }
              }
            }
          }
        }
      }
      if (q == 0 && lane == 0) {
        decode_trace(p, 9);
        if (local < 2) decode_trace(p, 10 + local);
      }
    }
    if (q == 0 && lane == 0) decode_trace(p, 14);
  }

  if (p.cluster > 1) {
    // Every thread of every CTA of the cluster takes every phase of the
    // cluster barrier exactly once, whatever path it took above: the set-up
    // phase (arrived at set-up; waited for before the first send, or here),
    // for the templates without a receive area of their own a phase after
    // which every partial is in its CTA's idle ring, and a last phase after
    // which every slice is in its finishing CTA's receive area (no CTA
    // touches another's shared memory after it).
    if constexpr (NH == 2) {  // the cluster form is never gated
      if (!cluster_waited) cluster_wait();  // the set-up phase
      uint32_t recv_s = base + S::OFF_RECV;
      if constexpr (!S::OWN_RECV) {
        cluster_sync();  // every partial in its CTA's idle ring
        if (threadIdx.x == 64) decode_trace(p, 6);
        recv_s = sW + S::RECV_OFF;
        if (warp >= 2) decode_cluster_push<MN, NH>(p, sW, recv_s);
        if (threadIdx.x == 64) decode_trace(p, 7);
      }
      cluster_sync();  // every slice in its finishing CTA's receive area
      if (threadIdx.x == 64) decode_trace(p, 8);
      // No CTA touches another's shared memory after this barrier.
      if (warp >= 2) decode_cluster_finish<MN, T, NH>(p, recv_s, cluster_bias);
      if (threadIdx.x == 64) decode_trace(p, 9);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, S::TMEM_COLS);
  }
  if (threadIdx.x == 0) decode_trace(p, 15);
}

}  // namespace dx
