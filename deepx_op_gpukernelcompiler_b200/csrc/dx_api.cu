// dx_api.cu — the C ABI declared in include/deepx_fused.h: argument checks,
// kernel selection, TMA descriptor encoding and launches.
//
// Behavioural contract mirrored from the reference engines
// (kernel_triton.py:70-89, kernel_tilelang.py:23-55): Y = act(X @ W + b) with
// an fp32 accumulator and the output in the input dtype.  Differences that
// the reference gets wrong and this library does not: ragged M/N are masked
// (kernel_triton.py:49-50 loads unmasked rows), the output keeps its true
// dtype (kernel_triton.py:65 always rounds to fp16), and GELU is selectable
// as tanh (the reference oracle, fusion.py:89) or erf (its kernels).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <new>
#include <string>
#include <utility>

#include "deepx_fused.h"
#include "dx_collective.cuh"
#include "dx_decode.cuh"
#include "dx_epilogue.cuh"
#include "dx_ptx.cuh"
#include "dx_simt.cuh"
#include "dx_umma_gemm.cuh"

namespace {

using dx::DecodeParams;
using dx::DecodeShape;
using dx::Umma2Shape;
using dx::UmmaParams;
using dx::UmmaShape;

thread_local std::string t_last_error;
thread_local std::string t_last_plan;

// Timeline buffer for the tensor-core kernels (dx_set_trace_buffer).
std::atomic<unsigned long long*> g_trace{nullptr};
std::atomic<size_t> g_trace_bytes{0};

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

void set_plan(const char* fmt, ...) {
  char buf[256];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_plan = buf;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(DX_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

// ------------------------------------------------------------ driver entry
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

bool load_encode_fn() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return g_encode != nullptr;
}

// Unique id of the calling thread's current CUDA context (0 if none is
// current yet).  Device-side state of this library — the module's __device__
// variables, function attributes — belongs to a context, and a device can
// have several over a process's life (cudaDeviceReset, or a caller's own
// context), so caches of that state are keyed by this id, which the driver
// never reuses within a process.
PFN_cuCtxGetCurrent_v4000 g_ctx_current = nullptr;
PFN_cuCtxGetId_v12000 g_ctx_id = nullptr;
std::once_flag g_ctx_once;

unsigned long long current_context_id() {
  std::call_once(g_ctx_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_ctx_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(fn);
    fn = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_ctx_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(fn);
  });
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (g_ctx_current == nullptr || g_ctx_id == nullptr || g_ctx_current(&ctx) != CUDA_SUCCESS ||
      ctx == nullptr || g_ctx_id(ctx, &id) != CUDA_SUCCESS)
    return 0;
  return id;
}

// --------------------------------------------------------- device facts
std::mutex g_mu;
std::map<int, int> g_sm_count;
std::map<std::pair<unsigned long long, const void*>, bool> g_attr_done;

int device_sms(int dev, int* sms) {
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_sm_count.find(dev);
  if (it != g_sm_count.end()) {
    *sms = it->second;
    return DX_OK;
  }
  int v = 0;
  cudaError_t e = cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(SM count)");
  g_sm_count[dev] = v;
  *sms = v;
  return DX_OK;
}

// SMs the launching stream may use: the whole device, or the SM partition of
// the green context the stream belongs to.  The persistent kernels size their
// grids to it (every CTA must be resident: the split-K pieces of a tile wait
// for one another), so they run correctly inside an SM partition.
PFN_cuStreamGetCtx_v12050 g_stream_ctx = nullptr;
PFN_cuGreenCtxGetDevResource_v12040 g_green_res = nullptr;
std::once_flag g_green_once;
std::map<CUgreenCtx, int> g_green_sms;

int stream_sms(cudaStream_t s, int dev, int* sms) {
  int rc = device_sms(dev, sms);
  if (rc) return rc;
  std::call_once(g_green_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuStreamGetCtx", &fn, 12050, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_stream_ctx = reinterpret_cast<PFN_cuStreamGetCtx_v12050>(fn);
    fn = nullptr;
    if (cudaGetDriverEntryPoint("cuGreenCtxGetDevResource", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_green_res = reinterpret_cast<PFN_cuGreenCtxGetDevResource_v12040>(fn);
  });
  (void)cudaGetLastError();
  if (g_stream_ctx == nullptr || g_green_res == nullptr) return DX_OK;
  CUcontext ctx = nullptr;
  CUgreenCtx green = nullptr;
  if (g_stream_ctx(reinterpret_cast<CUstream>(s), &ctx, &green) != CUDA_SUCCESS || green == nullptr)
    return DX_OK;  // a regular context: the whole device
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_green_sms.find(green);
  if (it == g_green_sms.end()) {
    CUdevResource r{};
    int n = *sms;
    if (g_green_res(green, &r, CU_DEV_RESOURCE_TYPE_SM) == CUDA_SUCCESS && r.sm.smCount > 0)
      n = static_cast<int>(r.sm.smCount);
    it = g_green_sms.emplace(green, n).first;
  }
  *sms = std::min(*sms, it->second);
  return DX_OK;
}

// ------------------------------------------------- timeout reporting
// One pinned, device-mapped int per device: the host-visible copy of the
// device status word (dx::g_status_mirror).  Installed on a device by the
// first call that is not being captured into a graph; afterwards every entry
// point reads its device's word before launching, without synchronising.
constexpr int kMaxDevices = 64;
int* g_host_status = nullptr;  // kMaxDevices words, pinned and mapped
std::map<unsigned long long, bool> g_mirror_installed;  // by context id

int install_status_mirror(int dev, cudaStream_t s) {
  if (dev < 0 || dev >= kMaxDevices) return DX_OK;
  const unsigned long long ctx = current_context_id();
  std::lock_guard<std::mutex> lk(g_mu);
  if (ctx != 0 && g_mirror_installed.count(ctx)) return DX_OK;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
    (void)cudaGetLastError();
    return DX_OK;  // set up by a later call outside the capture
  }
  if (g_host_status == nullptr) {
    void* h = nullptr;
    cudaError_t e = cudaHostAlloc(&h, kMaxDevices * sizeof(int),
                                  cudaHostAllocMapped | cudaHostAllocPortable);
    if (e != cudaSuccess) return cuda_fail(e, "cudaHostAlloc(status mirror)");
    std::memset(h, 0, kMaxDevices * sizeof(int));
    g_host_status = static_cast<int*>(h);
  }
  int* dptr = nullptr;
  cudaError_t e = cudaHostGetDevicePointer(reinterpret_cast<void**>(&dptr), g_host_status + dev, 0);
  if (e != cudaSuccess) return cuda_fail(e, "cudaHostGetDevicePointer(status mirror)");
  e = cudaMemcpyToSymbol(dx::g_status_mirror, &dptr, sizeof(dptr));
  if (e != cudaSuccess) return cuda_fail(e, "install status mirror");
  const unsigned long long now = current_context_id();  // the copy made one current
  if (now != 0) g_mirror_installed[now] = true;
  return DX_OK;
}

// DX_ERR_DEVICE_TIMEOUT when an earlier launch on `dev` reported a wait that
// ran out and dx_device_status has not cleared it since.
int check_status_mirror(int dev) {
  if (g_host_status == nullptr || dev < 0 || dev >= kMaxDevices) return DX_OK;
  if (reinterpret_cast<volatile int*>(g_host_status)[dev] == 0) return DX_OK;
  return fail(DX_ERR_DEVICE_TIMEOUT,
              "an earlier launch on device %d gave up a bounded wait, so its output is "
              "incomplete (and a split-K workspace may hold stale tickets); dx_device_status "
              "reads and clears the condition",
              dev);
}

int ensure_smem_attr(int dev, const void* fn, int smem_bytes, bool max_carveout) {
  (void)dev;
  const unsigned long long ctx = current_context_id();
  std::lock_guard<std::mutex> lk(g_mu);
  auto key = std::make_pair(ctx, fn);
  if (g_attr_done.count(key)) return DX_OK;
  cudaError_t e =
      cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(max dynamic smem)");
  if (max_carveout) {
    e = cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(carveout)");
  }
  if (ctx != 0) g_attr_done[key] = true;  // no context yet: set again next time
  return DX_OK;
}

// ------------------------------------------------------------- TMA maps
int make_tmap_2d(CUtensorMap* m, const void* ptr, CUtensorMapDataType dt, uint64_t inner,
                 uint64_t outer, uint64_t ld_elems, uint32_t box_inner, uint32_t box_outer,
                 CUtensorMapSwizzle sw, const char* name) {
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld_elems * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  CUresult r = g_encode(m, dt, 2, const_cast<void*>(ptr), dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(DX_ERR_CUDA, "cuTensorMapEncodeTiled(%s) failed with CUresult %d", name,
                static_cast<int>(r));
  return DX_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// A 16-bit matrix TMA can address: 16-byte-aligned base, row pitch a
// multiple of 16 bytes.
bool tma_ok(const void* p, int64_t ld) { return p != nullptr && aligned16(p) && (ld * 2) % 16 == 0; }

struct Problem {
  const void *X, *W, *bias, *R;
  void* Y;
  int64_t M, N, K, ldx, ldw, ldr, ldy;
  int dtype, act;
  void* ws;
  size_t ws_bytes;
  cudaStream_t stream;
  float alpha = 1.0f;  // Y = act(alpha * X W + bias) + R
  // Gated form: Y = act(X W + bias) * (X W2 + bias2); no residual, alpha 1.
  bool gated = false;
  const void* W2 = nullptr;
  const void* bias2 = nullptr;
  int64_t ldw2 = 0;
  // Row-parallel reduction job carried by a tensor-core launch (or run as a
  // standalone launch after the GEMM when another variant runs), or nullptr.
  const dx::RowReduceArgs* comm = nullptr;
  int comm_dtype = 0;
};

// ----------------------------------------------------------- decode plan
constexpr int kDecodeMaxM = 64;
constexpr int kDecodeTileN = 256;  // W columns per decode work unit
// Tickets live in a fixed slab at the start of every decode workspace, so the
// partial sums of one problem never overlap the tickets of another problem
// that reuses the same workspace later; the kernel leaves the slab zeroed.
constexpr size_t kTicketSlabBytes = size_t(64) << 10;
// (one 32-bit counter word per tile and warp quarter)
constexpr int64_t kDecodeMaxTiles = static_cast<int64_t>(kTicketSlabBytes / (4 * sizeof(int)));

int decode_mn(int64_t M) { return M <= 16 ? 16 : (M <= 32 ? 32 : 64); }

long long decode_cta_of_host(long long u, long long U, int G) {
  int g = static_cast<int>((u * G) / U);
  while (g + 1 < G && ((static_cast<long long>(g) + 1) * U) / G <= u) ++g;
  return g;
}

struct DecodePlan {
  int n_tiles = 0, kbt = 0, grid = 0, max_seg = 0, mn = 16;
  int nh = 2;  // 128-column UMMA halves per work unit
  int cluster = 1;  // CTAs per tile sharing partials in a thread-block cluster
  long long units = 0;
  size_t ticket_bytes = 0, bytes = 0;
};

// Thread-block cluster size for a plain decode problem whose tiles must be
// split along K: the largest C in {8, 4, 2} with tiles * C <= SMs and at least
// one k-block per CTA, provided tiles * C CTAs still cover half the SMs (so
// that enough SMs stream W); 1 when no such C exists.
int decode_cluster_size(int64_t n_tiles, int kbt, int sms) {
  for (int c : {8, 4, 2})
    if (n_tiles * c <= sms && kbt >= c && 2 * n_tiles * c >= sms) return c;
  return 1;
}

// Halves per work unit: 2; the gated form with M <= 16 uses 4 (256 columns
// of each weight, so both weights are read in 512-byte row segments).
// Whether a decode plan over tiles `tile_n` columns wide streams one whole
// tile per CTA (at least half as many tiles as SMs, at most one per SM).
bool decode_whole_tiles(int64_t N, int64_t tile_n, int sms) {
  const int64_t t = (N + tile_n - 1) / tile_n;
  return 2 * t >= sms && t <= sms;
}

// Halves per work unit: 2, or 4 for the gated form with M <= 16 (256 columns
// of each weight, 512-byte row segments) unless 128-column units give whole
// tiles and 256-column units do not (gated M = 16, K = 8192, N = 14336: 112
// whole tiles in 76 us against 56 split tiles in 84 us).
int decode_halves(int64_t M, int64_t N, int sms, bool gated) {
  if (!gated || decode_mn(M) != 16) return 2;
  return decode_whole_tiles(N, 128, sms) && !decode_whole_tiles(N, 256, sms) ? 2 : 4;
}

// Output columns per work unit: 256 (plain), 64 x halves (gated).
int decode_tile_n(int nh, bool gated) { return gated ? 64 * nh : kDecodeTileN; }

// Narrowest output tile of either halves choice: bounds the tile count.
int decode_min_tile_n(bool gated) { return gated ? 128 : kDecodeTileN; }

DecodePlan decode_plan(int64_t M, int64_t N, int64_t K, int sms, bool gated = false) {
  DecodePlan d;
  d.mn = decode_mn(M);
  d.nh = decode_halves(M, N, sms, gated);
  const int tile_n = decode_tile_n(d.nh, gated);
  d.n_tiles = static_cast<int>((N + tile_n - 1) / tile_n);
  d.kbt = static_cast<int>((K + 63) / 64);
  d.units = static_cast<long long>(d.n_tiles) * d.kbt;
  // One CTA per SM and an even split of the units, unless there are at
  // least half as many tiles as SMs: then one CTA streams each whole tile —
  // no split-K partials or fix-up, and those CTAs already saturate HBM
  // (M=16, N=28672, K=8192: 82.4 us with the split over 148 CTAs, 76.3 us
  // with 112 whole tiles).
  long long want = sms;
  if (2LL * d.n_tiles >= sms && d.n_tiles <= sms) want = d.n_tiles;
  d.ticket_bytes = kTicketSlabBytes;
  if (!gated && want == sms) {
    // Fewer tiles than SMs / 2: split each tile over a cluster of C CTAs that
    // add their partials through distributed shared memory (no workspace).
    const int c = decode_cluster_size(d.n_tiles, d.kbt, sms);
    if (c > 1) {
      d.cluster = c;
      d.grid = d.n_tiles * c;
      d.max_seg = c;
      d.bytes = 0;
      return d;
    }
  }
  d.grid = static_cast<int>(std::max<long long>(1, std::min<long long>(d.units, want)));
  int ms = 1;
  for (int t = 0; t < d.n_tiles; ++t) {
    const long long f = decode_cta_of_host(static_cast<long long>(t) * d.kbt, d.units, d.grid);
    const long long l =
        decode_cta_of_host(static_cast<long long>(t + 1) * d.kbt - 1, d.units, d.grid);
    ms = std::max<int>(ms, static_cast<int>(l - f + 1));
  }
  d.max_seg = ms;
  d.ticket_bytes = kTicketSlabBytes;
  // Whole tiles only (every tile streamed by one CTA): no tickets, no
  // partials, no workspace.
  d.bytes = ms == 1 ? 0
                    : d.ticket_bytes + static_cast<size_t>(d.n_tiles) * d.max_seg * d.mn *
                                           (128 * d.nh) * sizeof(float);
  return d;
}

// -------------------------------------------------------------- launches
CUtensorMapDataType tma_dtype(int dtype) {
  return dtype == DX_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
}

// Rows of X per raster group: keep group_m x rows x K x 2 bytes within ~48 MB
// (about a third of L2), with groups of equal size.
int pick_group_m(int m_tiles, int64_t rows_per_tile, int64_t K) {
  const int64_t panel = std::max<int64_t>(rows_per_tile * K * 2, 1);
  const int64_t max_g = std::max<int64_t>(1, (48LL << 20) / panel);
  const int64_t groups = (m_tiles + max_g - 1) / max_g;
  return static_cast<int>((m_tiles + groups - 1) / groups);
}

int make_umma_maps(const Problem& pr, CUtensorMap* tA, CUtensorMap* tB, CUtensorMap* tB2,
                   CUtensorMap* tY, CUtensorMap* tR) {
  const CUtensorMapDataType dt = tma_dtype(pr.dtype);
  int rc;
  if ((rc = make_tmap_2d(tA, pr.X, dt, pr.K, pr.M, pr.ldx, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B,
                         "X")))
    return rc;
  if ((rc = make_tmap_2d(tB, pr.W, dt, pr.N, pr.K, pr.ldw, 64, 64, CU_TENSOR_MAP_SWIZZLE_128B,
                         "W")))
    return rc;
  if (pr.gated) {
    if ((rc = make_tmap_2d(tB2, pr.W2, dt, pr.N, pr.K, pr.ldw2, 64, 64,
                           CU_TENSOR_MAP_SWIZZLE_128B, "W2")))
      return rc;
  } else {
    *tB2 = *tB;  // never read
  }
  if ((rc = make_tmap_2d(tY, pr.Y, dt, pr.N, pr.M, pr.ldy, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B,
                         "Y")))
    return rc;
  if (pr.R != nullptr) {
    if ((rc = make_tmap_2d(tR, pr.R, dt, pr.N, pr.M, pr.ldr, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B,
                           "R")))
      return rc;
  } else {
    *tR = *tY;  // never read: has_residual == 0
  }
  return DX_OK;
}

// ------------------------------------------------------------ UMMA plan
// One launch of a tensor-core GEMM: kernel (CTA pairs or single CTAs), tile
// width BN, and the schedule: full waves of whole tiles, then the tiles of
// the last partial wave split `splits` ways along K when a workspace allows.
struct UmmaPlan {
  bool pair = false;
  bool gated = false;  // output tiles bn / 2 wide, no split tail
  int bn = 256;
  int rows = 128;  // tile rows: 256 for pairs
  int workers = 0;
  int num_tiles = 0, dp_tiles = 0, splits = 1, k_blocks = 0;
  size_t bytes = 0;  // workspace bytes the plan needs (0: none)
};

// Relative throughput of each kernel/tile shape per SM, measured on B200
// (single-CTA 128x128 at 0.93 and the pair kernel at 256x128 at 0.80 of the
// pair kernel at 256x256).
double umma_efficiency(bool pair, int bn) {
  if (pair) return bn == 256 ? 1.00 : 0.80;
  return bn == 256 ? 0.97 : 0.93;
}

UmmaPlan plan_umma(int64_t M, int64_t N, int64_t K, int sms, int pair_slots, bool allow_split,
                   bool single_cta_only, bool gated = false) {
  UmmaPlan best;
  double best_cost = 1e300;
  const int kb = static_cast<int>((K + 63) / 64);
  if (gated) allow_split = false;
  for (int use_pair = 0; use_pair < 2; ++use_pair) {
    if (use_pair && (single_cta_only || M < 256 || pair_slots <= 0)) continue;
    for (int bn : {256, 128}) {
      // The gated kernels exist for BN = 256 (128 gate + 128 up columns).
      if (gated ? bn != 256 : (bn == 256 && N <= 128)) continue;
      UmmaPlan pl;
      pl.pair = use_pair != 0;
      pl.gated = gated;
      pl.bn = bn;
      pl.rows = pl.pair ? 256 : 128;
      pl.workers = pl.pair ? pair_slots : sms;
      pl.k_blocks = kb;
      const int64_t tile_n = gated ? bn / 2 : bn;
      const int64_t tiles = ((M + pl.rows - 1) / pl.rows) * ((N + tile_n - 1) / tile_n);
      pl.num_tiles = static_cast<int>(tiles);
      const int64_t full = tiles / pl.workers, rem = tiles % pl.workers;
      int splits = 1;
      if (allow_split && rem > 0) {
        // Each piece finishes a share of the tile's 32-column chunks, so at
        // most BN / 32 pieces; each piece keeps at least 8 k-blocks.
        splits = static_cast<int>(
            std::min<int64_t>(std::min<int64_t>(pl.workers / rem, kb / 8), bn / 32));
        if (splits < 2) splits = 1;
      }
      pl.splits = splits;
      pl.dp_tiles = splits > 1 ? static_cast<int>(tiles - rem) : pl.num_tiles;
      pl.bytes = splits > 1 ? kTicketSlabBytes + static_cast<size_t>(rem) * splits *
                                                     (pl.pair ? 2 : 1) * 128 * bn * sizeof(float)
                            : 0;
      const double tail = rem == 0 ? 0.0 : (splits > 1 ? 1.0 / splits + 0.05 : 1.0);
      const double cost = (static_cast<double>(full) + tail) * bn / umma_efficiency(pl.pair, bn);
      if (cost < best_cost) {
        best_cost = cost;
        best = pl;
      }
    }
  }
  return best;
}

UmmaParams umma_params(const Problem& pr, const UmmaPlan& pl) {
  UmmaParams p{};
  p.M = static_cast<int>(pr.M);
  p.N = static_cast<int>(pr.N);
  p.K = static_cast<int>(pr.K);
  p.m_tiles = static_cast<int>((pr.M + pl.rows - 1) / pl.rows);
  const int tile_n = pl.gated ? pl.bn / 2 : pl.bn;
  p.n_tiles = static_cast<int>((pr.N + tile_n - 1) / tile_n);
  p.k_blocks = pl.k_blocks;
  p.num_tiles = p.m_tiles * p.n_tiles;
  p.group_m = pick_group_m(p.m_tiles, pl.rows, pr.K);
  p.bias = pr.bias;
  p.bias2 = pr.bias2;
  p.act = pr.act;
  p.has_residual = pr.R != nullptr ? 1 : 0;
  p.alpha = pr.alpha;
  p.workers = pl.workers;
  p.dp_tiles = pl.dp_tiles;
  p.splits = pl.splits;
  p.tickets = pl.splits > 1 ? static_cast<int*>(pr.ws) : nullptr;
  {
    unsigned long long* tr = g_trace.load();
    const size_t need = static_cast<size_t>(pl.workers) * (pl.pair ? 2 : 1) * dx::kTraceSlots * 8;
    p.trace = (tr != nullptr && g_trace_bytes.load() >= need) ? tr : nullptr;
  }
  p.partials = pl.splits > 1
                   ? reinterpret_cast<float*>(static_cast<char*>(pr.ws) + kTicketSlabBytes)
                   : nullptr;
  p.comm_on = pr.comm != nullptr ? 1 : 0;
  if (pr.comm != nullptr) p.comm = *pr.comm;
  return p;
}

// Launch grid: no more workers than work items.
int umma_grid_workers(const UmmaPlan& pl) {
  const int64_t items = static_cast<int64_t>(pl.dp_tiles) +
                        static_cast<int64_t>(pl.num_tiles - pl.dp_tiles) * pl.splits;
  return static_cast<int>(std::min<int64_t>(pl.workers, items));
}

// Programmatic dependent launch for the persistent GEMM and decode kernels
// (they wait for the preceding grid before touching global memory, so their
// set-up overlaps its tail).  DX_PDL=0 in the environment turns it off.
bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("DX_PDL");
    return v == nullptr || std::strcmp(v, "0") != 0;
  }();
  return on;
}

// Launch configuration with an optional cluster size (cluster <= 1: none)
// and, when `pdl` and pdl_enabled(), the programmatic-serialization
// attribute; `attr` holds >= 2 entries.
cudaLaunchConfig_t launch_config(int grid, int threads, int smem, cudaStream_t s, int cluster,
                                 cudaLaunchAttribute* attr, bool pdl = true) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(static_cast<unsigned>(threads));
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = s;
  unsigned n = 0;
  if (cluster > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = static_cast<unsigned>(cluster);
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  if (pdl && pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cfg;
}

template <int BN, typename T, bool G = false>
int launch_umma(const Problem& pr, int dev, const UmmaPlan& pl) {
  using S = UmmaShape<BN>;
  auto kern = dx::umma_fused_linear_kernel<BN, T, G>;
  int rc = ensure_smem_attr(dev, reinterpret_cast<const void*>(kern), S::SMEM_BYTES, false);
  if (rc) return rc;
  CUtensorMap tA, tB, tB2, tY, tR;
  if ((rc = make_umma_maps(pr, &tA, &tB, &tB2, &tY, &tR))) return rc;
  const UmmaParams p = umma_params(pr, pl);
  const int grid = umma_grid_workers(pl);
  set_plan("umma_1cta%s tile=128x%d stages=%d grid=%d tiles=%d dp_tiles=%d splits=%d group_m=%d "
           "smem=%d workspace=%zu",
           G ? "_gated" : "", G ? BN / 2 : BN, S::STAGES, grid, p.num_tiles, p.dp_tiles, p.splits,
           p.group_m, S::SMEM_BYTES, pl.bytes);
  // Tracing writes timestamps before the grid dependency wait: no early start.
  cudaLaunchAttribute attr[2];
  cudaLaunchConfig_t cfg =
      launch_config(grid, S::THREADS, S::SMEM_BYTES, pr.stream, 1, attr, p.trace == nullptr);
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tA, tB, tB2, tY, tR, p);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch umma_fused_linear_kernel");
  return DX_OK;
}

cudaLaunchConfig_t pair_launch_config(int grid, int threads, int smem, cudaStream_t s,
                                      cudaLaunchAttribute* attr) {
  return launch_config(grid, threads, smem, s, 2, attr);
}

std::map<int, int> g_pair_slots;

// How many CTA pairs of the pair kernel can be resident at once (cached per
// device; the pair kernels share one shared-memory footprint class).
template <int BN, typename T>
int pair_slots(int dev, int sms) {
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_pair_slots.find(dev);
    if (it != g_pair_slots.end()) return it->second;
  }
  using S = Umma2Shape<BN>;
  auto kern = dx::umma2_fused_linear_kernel<BN, T>;
  if (ensure_smem_attr(dev, reinterpret_cast<const void*>(kern), S::SMEM_BYTES, false) != DX_OK)
    return 0;
  cudaLaunchAttribute attr[2];
  cudaLaunchConfig_t cfg = pair_launch_config(2 * (sms / 2), S::THREADS, S::SMEM_BYTES, nullptr, attr);
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, reinterpret_cast<const void*>(kern), &cfg) != cudaSuccess)
    n = 0;
  (void)cudaGetLastError();
  std::lock_guard<std::mutex> lk(g_mu);
  g_pair_slots[dev] = n;
  return n;
}

template <int BN, typename T, bool G = false>
int launch_umma2(const Problem& pr, int dev, const UmmaPlan& pl) {
  using S = Umma2Shape<BN>;
  auto kern = dx::umma2_fused_linear_kernel<BN, T, G>;
  int rc = ensure_smem_attr(dev, reinterpret_cast<const void*>(kern), S::SMEM_BYTES, false);
  if (rc) return rc;
  CUtensorMap tA, tB, tB2, tY, tR;
  if ((rc = make_umma_maps(pr, &tA, &tB, &tB2, &tY, &tR))) return rc;
  const UmmaParams p = umma_params(pr, pl);
  const int grid = 2 * umma_grid_workers(pl);
  set_plan("umma_pair%s tile=256x%d stages=%d grid=%d pair_slots=%d tiles=%d dp_tiles=%d "
           "splits=%d group_m=%d smem=%d workspace=%zu",
           G ? "_gated" : "", G ? BN / 2 : BN, S::STAGES, grid, pl.workers, p.num_tiles,
           p.dp_tiles, p.splits, p.group_m, S::SMEM_BYTES, pl.bytes);
  cudaLaunchAttribute attr[2];
  cudaLaunchConfig_t cfg =
      launch_config(grid, S::THREADS, S::SMEM_BYTES, pr.stream, 2, attr, p.trace == nullptr);
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tA, tB, tB2, tY, tR, p);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch umma2_fused_linear_kernel");
  return DX_OK;
}

// Largest weight stream (bytes) for which a decode launch starts early.
constexpr int64_t kDecodePdlMaxBytes = int64_t{160} << 20;

template <int MN, typename T, int NH = 2>
int launch_decode(const Problem& pr, int dev, int sms, const DecodePlan& d) {
  using S = DecodeShape<MN, NH>;
  auto kern = dx::decode_fused_linear_kernel<MN, T, NH>;
  int rc = ensure_smem_attr(dev, reinterpret_cast<const void*>(kern), S::SMEM_BYTES, true);
  if (rc) return rc;
  const CUtensorMapDataType dt = tma_dtype(pr.dtype);
  CUtensorMap tW, tW2, tX;
  if ((rc = make_tmap_2d(&tW, pr.W, dt, pr.N, pr.K, pr.ldw, 64, 64, CU_TENSOR_MAP_SWIZZLE_128B,
                         "W")))
    return rc;
  if (pr.gated) {
    if ((rc = make_tmap_2d(&tW2, pr.W2, dt, pr.N, pr.K, pr.ldw2, 64, 64,
                           CU_TENSOR_MAP_SWIZZLE_128B, "W2")))
      return rc;
  } else {
    tW2 = tW;  // never read
  }
  if ((rc = make_tmap_2d(&tX, pr.X, dt, pr.K, pr.M, pr.ldx, 64, MN, CU_TENSOR_MAP_SWIZZLE_128B,
                         "X")))
    return rc;
  DecodeParams p{};
  p.M = static_cast<int>(pr.M);
  p.N = static_cast<int>(pr.N);
  p.K = static_cast<int>(pr.K);
  p.n_tiles = d.n_tiles;
  p.kbt = d.kbt;
  p.units = d.units;
  p.grid = d.grid;
  p.max_seg = d.max_seg;
  p.ldy = pr.ldy;
  p.ldr = pr.ldr;
  p.bias = pr.bias;
  p.residual = pr.R;
  p.Y = pr.Y;
  // Unused by whole-tile plans (max_seg == 1), which may run without a workspace.
  p.tickets = pr.ws != nullptr ? static_cast<int*>(pr.ws) : nullptr;
  p.partials = pr.ws != nullptr
                   ? reinterpret_cast<float*>(static_cast<char*>(pr.ws) + d.ticket_bytes)
                   : nullptr;
  p.act = pr.act;
  p.alpha = pr.alpha;
  p.gated = pr.gated ? 1 : 0;
  p.bias2 = pr.bias2;
  p.cluster = d.cluster;
  {
    unsigned long long* tr = g_trace.load();
    const size_t need = static_cast<size_t>(d.grid) * dx::kTraceSlots * 8;
    p.trace = (tr != nullptr && g_trace_bytes.load() >= need) ? tr : nullptr;
  }
  (void)sms;
  set_plan("decode%s mn=%d halves=%d stages=%d grid=%d n_tiles=%d kbt=%d max_seg=%d "
           "cluster=%d workspace=%zu",
           pr.gated ? "_gated" : "", MN, NH, S::STAGES, d.grid, d.n_tiles, d.kbt, d.max_seg,
           d.cluster, d.bytes);
  // An early start gains the set-up time (barriers, TMEM, descriptor
  // prefetch), a few microseconds; a long weight stream loses more than that
  // to the uneven SM placement of CTAs that start while the previous grid
  // still holds SMs (measured: 16x8192x3584 f16 18.2 -> 15.8 us, but
  // 16x8192x28672 1.7% slower), so only short launches take it.  Tracing
  // writes timestamps before the wait: no early start.
  const int64_t w_bytes = pr.K * pr.N * (pr.gated ? 2 : 1) * static_cast<int64_t>(sizeof(T));
  cudaLaunchAttribute attr[2];
  cudaLaunchConfig_t cfg = launch_config(d.grid, S::THREADS, S::SMEM_BYTES, pr.stream, d.cluster,
                                         attr, p.trace == nullptr && w_bytes <= kDecodePdlMaxBytes);
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tW, tW2, tX, p);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch decode_fused_linear_kernel");
  return DX_OK;
}

template <typename T>
int launch_simt(const Problem& pr, int sms) {
  const T* X = static_cast<const T*>(pr.X);
  const T* W = static_cast<const T*>(pr.W);
  const T* b = static_cast<const T*>(pr.bias);
  const T* R = static_cast<const T*>(pr.R);
  T* Y = static_cast<T*>(pr.Y);
  const int M = static_cast<int>(pr.M), N = static_cast<int>(pr.N), K = static_cast<int>(pr.K);
  // The largest tile that still gives at least two CTAs per SM (64x64, 32x32,
  // 16x32); below that, the smallest.
  const int64_t t64 = ((pr.M + 63) / 64) * ((pr.N + 63) / 64);
  const int64_t t32 = ((pr.M + 31) / 32) * ((pr.N + 31) / 32);
  const int bm = t64 >= 2LL * sms ? 64 : (t32 >= 2LL * sms ? 32 : 16);
  const int bn = bm == 16 ? 32 : bm;
  if ((pr.M + bm - 1) / bm > 65535) return fail(DX_ERR_UNSUPPORTED, "M too large for the SIMT kernel");
  dim3 grid(static_cast<unsigned>((pr.N + bn - 1) / bn), static_cast<unsigned>((pr.M + bm - 1) / bm));
  set_plan("simt tile=%dx%d grid=%u", bm, bn, grid.x * grid.y);
  if (bm == 64)
    dx::simt_fused_linear_kernel<T, 64, 64, 32><<<grid, 256, 0, pr.stream>>>(
        X, W, b, R, Y, M, N, K, pr.ldx, pr.ldw, pr.ldr, pr.ldy, pr.act, pr.alpha);
  else if (bm == 32)
    dx::simt_fused_linear_kernel<T, 32, 32, 128><<<grid, 256, 0, pr.stream>>>(
        X, W, b, R, Y, M, N, K, pr.ldx, pr.ldw, pr.ldr, pr.ldy, pr.act, pr.alpha);
  else
    dx::simt_fused_linear_kernel<T, 16, 32, 128><<<grid, 256, 0, pr.stream>>>(
        X, W, b, R, Y, M, N, K, pr.ldx, pr.ldw, pr.ldr, pr.ldy, pr.act, pr.alpha);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch simt_fused_linear_kernel");
  return DX_OK;
}

template <typename T>
int launch_simt_gated(const Problem& pr, int sms) {
  const T* X = static_cast<const T*>(pr.X);
  const T* Wg = static_cast<const T*>(pr.W);
  const T* Wu = static_cast<const T*>(pr.W2);
  const T* bg = static_cast<const T*>(pr.bias);
  const T* bu = static_cast<const T*>(pr.bias2);
  T* Y = static_cast<T*>(pr.Y);
  const int M = static_cast<int>(pr.M), N = static_cast<int>(pr.N), K = static_cast<int>(pr.K);
  const bool big = ((pr.M + 63) / 64) * ((pr.N + 63) / 64) >= 2LL * sms;
  const int tile = big ? 64 : 32;
  if ((pr.M + tile - 1) / tile > 65535) return fail(DX_ERR_UNSUPPORTED, "M too large for the SIMT kernel");
  dim3 grid(static_cast<unsigned>((pr.N + tile - 1) / tile),
            static_cast<unsigned>((pr.M + tile - 1) / tile));
  set_plan("simt_gated tile=%d grid=%ux%u", tile, grid.x, grid.y);
  if (big)
    dx::simt_gated_linear_kernel<T, 64, 64><<<grid, 256, 0, pr.stream>>>(
        X, Wg, Wu, bg, bu, Y, M, N, K, pr.ldx, pr.ldw, pr.ldw2, pr.ldy, pr.act);
  else
    dx::simt_gated_linear_kernel<T, 32, 32><<<grid, 256, 0, pr.stream>>>(
        X, Wg, Wu, bg, bu, Y, M, N, K, pr.ldx, pr.ldw, pr.ldw2, pr.ldy, pr.act);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch simt_gated_linear_kernel");
  return DX_OK;
}

// ---------------------------------------------------------- validation
int validate(const Problem& p, int kernel) {
  if (p.dtype < DX_DTYPE_F32 || p.dtype > DX_DTYPE_BF16)
    return fail(DX_ERR_INVALID_ARGUMENT, "unknown dtype %d", p.dtype);
  if (p.act < DX_ACT_NONE || p.act > DX_ACT_SILU)
    return fail(DX_ERR_INVALID_ARGUMENT, "unknown activation %d", p.act);
  if (kernel < DX_KERNEL_AUTO || kernel > DX_KERNEL_UMMA_1CTA)
    return fail(DX_ERR_INVALID_ARGUMENT, "unknown kernel variant %d", kernel);
  if (p.M < 0 || p.N < 0 || p.K < 0)
    return fail(DX_ERR_INVALID_ARGUMENT, "negative shape M=%lld N=%lld K=%lld", (long long)p.M,
                (long long)p.N, (long long)p.K);
  const int64_t kMax = 0x7fffffffLL;
  if (p.M > kMax || p.N > kMax || p.K > kMax)
    return fail(DX_ERR_UNSUPPORTED, "dimension above 2^31-1");
  if (p.M == 0 || p.N == 0) return DX_OK;
  if (p.Y == nullptr) return fail(DX_ERR_INVALID_ARGUMENT, "Y is NULL");
  if (p.K > 0 && (p.X == nullptr || p.W == nullptr))
    return fail(DX_ERR_INVALID_ARGUMENT, "X or W is NULL");
  if (p.ldx < std::max<int64_t>(p.K, 1))
    return fail(DX_ERR_INVALID_ARGUMENT, "ldx=%lld < K=%lld", (long long)p.ldx, (long long)p.K);
  if (p.ldw < p.N)
    return fail(DX_ERR_INVALID_ARGUMENT, "ldw=%lld < N=%lld", (long long)p.ldw, (long long)p.N);
  if (p.ldy < p.N)
    return fail(DX_ERR_INVALID_ARGUMENT, "ldy=%lld < N=%lld", (long long)p.ldy, (long long)p.N);
  if (p.R != nullptr && p.ldr < p.N)
    return fail(DX_ERR_INVALID_ARGUMENT, "ldr=%lld < N=%lld", (long long)p.ldr, (long long)p.N);
  if (p.gated) {
    if (p.K > 0 && p.W2 == nullptr) return fail(DX_ERR_INVALID_ARGUMENT, "Wu is NULL");
    if (p.ldw2 < p.N)
      return fail(DX_ERR_INVALID_ARGUMENT, "ldwu=%lld < N=%lld", (long long)p.ldw2, (long long)p.N);
  }
  return DX_OK;
}

bool umma_eligible(const Problem& p) {
  if (p.dtype == DX_DTYPE_F32 || p.K == 0) return false;
  if (!tma_ok(p.X, p.ldx) || !tma_ok(p.W, p.ldw) || !tma_ok(p.Y, p.ldy)) return false;
  if (p.gated && !tma_ok(p.W2, p.ldw2)) return false;
  if (p.R != nullptr && !tma_ok(p.R, p.ldr)) return false;
  return true;
}

bool decode_eligible(const Problem& p) {
  if (p.dtype == DX_DTYPE_F32 || p.K == 0 || p.M > kDecodeMaxM) return false;
  const int tn = decode_min_tile_n(p.gated);
  if ((p.N + tn - 1) / tn > kDecodeMaxTiles) return false;
  if (p.gated && !tma_ok(p.W2, p.ldw2)) return false;
  return tma_ok(p.X, p.ldx) && tma_ok(p.W, p.ldw);
}

// Skinny-M problems the decode kernel streams faster than the single-CTA
// tensor-core kernel, measured on B200 (fp16, K = 4096 and 8192, N = 1792 to
// 28672, M = 1 to 64; `bench.py --skinny`):
//   * gated: up to M = 32; 32 < M <= 64 with narrow W (fewer than 20
//     256-column tiles) or K >= 8192 (K = 8192, N = 7168, M = 64: 58 us
//     against 64).  With K = 4096 and wide W the tensor-core kernel streams
//     both weights faster (N = 7168: 37 us against 41).
//   * plain, M < 16: always (below 8 rows the tensor-core kernel's TMA path is
//     slow, and rows that fill part of an 8-row group cost it too: M = 12,
//     K = 4096, N = 3584: 21 us against 31).
//   * plain, M = 16: with at least 20 tiles, or with K * N >= 2^23; only the
//     smallest W goes to the tensor-core kernel (K = 4096, N = 1792: 19 us
//     against 23, where the decode kernel's split-K fix-up dominates).
//   * plain, 16 < M <= 32: when W has at least half as many 256-column tiles
//     as SMs (one whole tile per CTA).
// For plain problems with 32 < M <= 64 the tensor-core kernel's 128-row tiles
// stream W faster (M = 64, N = 28672, K = 8192: 84 us against 91).
bool decode_preferred(int64_t M, int64_t N, int64_t K, int sms, bool gated) {
  const int mn = decode_mn(M);
  const int64_t n_tiles = (N + kDecodeTileN - 1) / kDecodeTileN;
  if (gated) return mn <= 32 || n_tiles < 20 || K >= 8192;
  if (mn == 16) return M < 16 || n_tiles >= 20 || K * N >= (int64_t(1) << 23);
  if (mn == 32) return 2 * n_tiles >= sms;
  return false;
}

int select_variant(const Problem& p, int sms, bool ws_known) {
  if (p.dtype == DX_DTYPE_F32 || p.K == 0) return DX_KERNEL_SIMT;
  if (decode_eligible(p) && (decode_preferred(p.M, p.N, p.K, sms, p.gated) || !umma_eligible(p))) {
    if (!ws_known) return DX_KERNEL_DECODE;
    const DecodePlan d = decode_plan(p.M, p.N, p.K, sms, p.gated);
    if (d.bytes == 0 || (p.ws != nullptr && p.ws_bytes >= d.bytes && aligned16(p.ws)))
      return DX_KERNEL_DECODE;
  }
  if (umma_eligible(p)) return DX_KERNEL_UMMA;
  return DX_KERNEL_SIMT;
}

// The plan for this call: with the split tail when the caller's workspace
// holds it, else whole tiles only.
UmmaPlan umma_plan_for(const Problem& p, int dev, int sms, bool single_cta_only) {
  const int slots = (p.M >= 256 && !single_cta_only)
                        ? std::min(pair_slots<256, __nv_bfloat16>(dev, sms), sms / 2)
                        : 0;
  UmmaPlan pl = plan_umma(p.M, p.N, p.K, sms, slots, true, single_cta_only, p.gated);
  if (pl.bytes > 0 && (p.ws == nullptr || p.ws_bytes < pl.bytes || !aligned16(p.ws)))
    pl = plan_umma(p.M, p.N, p.K, sms, slots, false, single_cta_only, p.gated);
  return pl;
}

template <typename T>
int dispatch_typed(const Problem& p, int variant, int dev, int sms) {
  switch (variant) {
    case DX_KERNEL_UMMA:
    case DX_KERNEL_UMMA_1CTA: {
      const UmmaPlan pl = umma_plan_for(p, dev, sms, variant == DX_KERNEL_UMMA_1CTA);
      if (p.gated)
        return pl.pair ? launch_umma2<256, T, true>(p, dev, pl) : launch_umma<256, T, true>(p, dev, pl);
      if (pl.pair)
        return pl.bn == 256 ? launch_umma2<256, T>(p, dev, pl) : launch_umma2<128, T>(p, dev, pl);
      return pl.bn == 256 ? launch_umma<256, T>(p, dev, pl) : launch_umma<128, T>(p, dev, pl);
    }
    case DX_KERNEL_DECODE: {
      const DecodePlan d = decode_plan(p.M, p.N, p.K, sms, p.gated);
      if (d.mn == 16)
        return d.nh == 4 ? launch_decode<16, T, 4>(p, dev, sms, d) : launch_decode<16, T>(p, dev, sms, d);
      if (d.mn == 32) return launch_decode<32, T>(p, dev, sms, d);
      return launch_decode<64, T>(p, dev, sms, d);
    }
    default:
      return p.gated ? launch_simt_gated<T>(p, sms) : launch_simt<T>(p, sms);
  }
}

// ------------------------------------------------ row-parallel reduction
// Checks a dx_row_reduce_job and fills the kernels' argument block.
int row_job_args(const dx_row_reduce_job* j, dx::RowReduceArgs* a) {
  if (j == nullptr || j->Y == nullptr)
    return fail(DX_ERR_INVALID_ARGUMENT, "row_reduce: NULL job or output");
  const int world = j->world, rank = j->rank;
  const int64_t M = j->M, N = j->N;
  if (world < 1 || world > dx::kRowMaxWorld || rank < 0 || rank >= world)
    return fail(DX_ERR_INVALID_ARGUMENT, "row_reduce: world must be 1..%d and 0 <= rank < world",
                dx::kRowMaxWorld);
  if (j->dtype != DX_DTYPE_F16 && j->dtype != DX_DTYPE_BF16)
    return fail(DX_ERR_UNSUPPORTED, "row_reduce supports fp16/bf16");
  if (M <= 0 || M % world != 0 || M > 0x7fffffffLL || N <= 0 || N % 8 != 0 || N > 0x7fffffffLL)
    return fail(DX_ERR_INVALID_ARGUMENT,
                "row_reduce needs M > 0 divisible by world (M=%lld, world=%d) and N %% 8 == 0",
                (long long)M, world);
  if (j->ldp < N || j->ldp % 8 != 0 || j->ldy < N || j->ldy % 8 != 0 ||
      (j->R != nullptr && (j->ldr < N || j->ldr % 8 != 0)))
    return fail(DX_ERR_INVALID_ARGUMENT, "row_reduce: pitches must be >= N and multiples of 8");
  if (j->epoch <= 0) return fail(DX_ERR_INVALID_ARGUMENT, "row_reduce: epoch must be positive");
  auto bad_chunk = [&](int64_t row0, int64_t rows, int chunk) {
    return rows < 0 || (rows > 0 && (row0 < 0 || row0 % world != 0 || rows % world != 0 ||
                                     row0 + rows > M || chunk < 0 ||
                                     chunk >= dx::kRowMaxChunks));
  };
  if (bad_chunk(j->a_row0, j->a_rows, j->a_chunk) || bad_chunk(j->b_row0, j->b_rows, j->b_chunk))
    return fail(DX_ERR_INVALID_ARGUMENT,
                "row_reduce: a chunk must lie in [0, M), start and span multiples of world, "
                "and have an index below %d",
                dx::kRowMaxChunks);
  if ((j->bias != nullptr && !aligned16(j->bias)) || (j->R != nullptr && !aligned16(j->R)) ||
      !aligned16(j->Y))
    return fail(DX_ERR_INVALID_ARGUMENT, "row_reduce needs 16-byte-aligned bias, R and Y");
  const bool nvls = j->mc_part != nullptr;
  if (nvls && (j->mc_out == nullptr || j->out_sym == nullptr || !aligned16(j->mc_part) ||
               !aligned16(j->mc_out) || !aligned16(j->out_sym) || j->ldo < N || j->ldo % 8 != 0))
    return fail(DX_ERR_INVALID_ARGUMENT,
                "row_reduce (multicast): mc_out and out_sym must be 16-byte aligned and ldo a "
                "multiple of 8 no smaller than N");
  *a = dx::RowReduceArgs{};
  for (int r = 0; r < world; ++r) {
    if (j->P[r] == nullptr || !aligned16(j->P[r]) ||
        (!nvls && (j->S[r] == nullptr || !aligned16(j->S[r]))) ||
        j->F[r] == nullptr || (reinterpret_cast<uintptr_t>(j->F[r]) & 3u) != 0)
      return fail(DX_ERR_INVALID_ARGUMENT, "row_reduce: buffers of rank %d NULL or misaligned", r);
    a->P.p[r] = j->P[r];
    a->S.p[r] = j->S[r];
    a->F.p[r] = j->F[r];
  }
  a->world = world;
  a->rank = rank;
  a->N = static_cast<int>(N);
  a->ldp = j->ldp;
  a->ldr = j->ldr;
  a->ldy = j->ldy;
  a->slab_base = static_cast<long long>(j->epoch & 1) * (M / world);
  a->a_row0 = j->a_row0;
  a->a_rows = static_cast<int>(j->a_rows);
  a->a_chunk = j->a_chunk;
  a->b_row0 = j->b_row0;
  a->b_rows = static_cast<int>(j->b_rows);
  a->b_chunk = j->b_chunk;
  a->bias = j->bias;
  a->R = j->R;
  a->Y = j->Y;
  a->epoch = j->epoch;
  a->mc_part = j->mc_part;
  a->mc_out = nvls ? j->mc_out : nullptr;
  a->out_sym = nvls ? j->out_sym : nullptr;
  a->ldo = nvls ? j->ldo : 0;
  return DX_OK;
}

// The standalone reduction kernel (one 512-thread CTA per SM by default).
int launch_row_reduce(const dx::RowReduceArgs& a, int dtype, int sms, int grid,
                      cudaStream_t s) {
  if (a.a_rows == 0 && a.b_rows == 0) return DX_OK;
  if (grid <= 0 || grid > dx::kRowCtasPerSm * sms) grid = dx::kRowCtasPerSm * sms;
  set_plan("row_reduce world=%d rank=%d A=[%lld,+%d) B=[%lld,+%d) N=%d grid=%d epoch=%d",
           a.world, a.rank, a.a_row0, a.a_rows, a.b_row0, a.b_rows, a.N, grid, a.epoch);
  if (dtype == DX_DTYPE_F16)
    dx::row_reduce_kernel<__half><<<grid, dx::kRowThreads, 0, s>>>(a);
  else
    dx::row_reduce_kernel<__nv_bfloat16><<<grid, dx::kRowThreads, 0, s>>>(a);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch row_reduce_kernel");
  return DX_OK;
}

int run(const Problem& p, int kernel) {
  t_last_error.clear();
  int rc = validate(p, kernel);
  if (rc) return rc;
  if (p.comm != nullptr && p.comm_dtype != p.dtype)
    return fail(DX_ERR_INVALID_ARGUMENT, "row_reduce job dtype differs from the GEMM's");
  if ((p.M == 0 || p.N == 0) && p.comm == nullptr) return DX_OK;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  int sms = 0;
  if ((rc = stream_sms(p.stream, dev, &sms))) return rc;
  if ((rc = install_status_mirror(dev, p.stream))) return rc;
  if ((rc = check_status_mirror(dev))) return rc;
  if (p.M == 0 || p.N == 0) return launch_row_reduce(*p.comm, p.comm_dtype, sms, 0, p.stream);

  int variant = kernel == DX_KERNEL_AUTO ? select_variant(p, sms, true) : kernel;
  if (variant == DX_KERNEL_UMMA || variant == DX_KERNEL_UMMA_1CTA || variant == DX_KERNEL_DECODE) {
    if (!load_encode_fn())
      return fail(DX_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  }
  if ((variant == DX_KERNEL_UMMA || variant == DX_KERNEL_UMMA_1CTA) && !umma_eligible(p))
    return fail(DX_ERR_UNSUPPORTED,
                "tcgen05 kernel needs fp16/bf16, K > 0, 16-byte-aligned pointers and row "
                "pitches that are multiples of 16 bytes");
  if (variant == DX_KERNEL_DECODE) {
    if (!decode_eligible(p))
      return fail(DX_ERR_UNSUPPORTED,
                  "decode kernel needs fp16/bf16, 0 < K, M <= %d, N <= %lld, and "
                  "16-byte-aligned X/W with row pitches that are multiples of 16 bytes",
                  kDecodeMaxM, (long long)(kDecodeMaxTiles * kDecodeTileN));
    const DecodePlan d = decode_plan(p.M, p.N, p.K, sms, p.gated);
    if (d.bytes > 0 && (p.ws == nullptr || p.ws_bytes < d.bytes || !aligned16(p.ws)))
      return fail(DX_ERR_WORKSPACE, "decode kernel needs a 16-byte-aligned workspace of %zu bytes",
                  d.bytes);
  }
  switch (p.dtype) {
    case DX_DTYPE_F32:
      if (variant != DX_KERNEL_SIMT)
        return fail(DX_ERR_UNSUPPORTED, "fp32 runs only on the exact-fp32 SIMT kernel");
      rc = p.gated ? launch_simt_gated<float>(p, sms) : launch_simt<float>(p, sms);
      break;
    case DX_DTYPE_F16:
      rc = dispatch_typed<__half>(p, variant, dev, sms);
      break;
    default:
      rc = dispatch_typed<__nv_bfloat16>(p, variant, dev, sms);
  }
  // Only the tensor-core kernels carry a job; after another variant it runs
  // as its own launch, stream-ordered after the GEMM.
  const bool carried = variant == DX_KERNEL_UMMA || variant == DX_KERNEL_UMMA_1CTA;
  if (rc == DX_OK && p.comm != nullptr && !carried) {
    const std::string gemm_plan = t_last_plan;
    rc = launch_row_reduce(*p.comm, p.comm_dtype, sms, 0, p.stream);
    if (rc == DX_OK) set_plan("%s +row_reduce launch", gemm_plan.c_str());
  } else if (rc == DX_OK && p.comm != nullptr) {
    const std::string gemm_plan = t_last_plan;
    set_plan("%s +row_reduce job A=%d B=%d", gemm_plan.c_str(), p.comm->a_rows, p.comm->b_rows);
  }
  return rc;
}

// One CTA waits, through the kernels' bounded mbarrier wait, on a barrier
// that nothing completes: after kWaitLimitNs the wait gives up, raises the
// device status word and the thread records 2 in *result (1 had the wait
// completed).  Exercises the failure path without a fault or a hang.
__global__ void selftest_wait_kernel(int* result) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    dx::mbar_init(dx::smem_u32(&bar), 1);
    abort_flag = 0;
    dx::fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const bool ok = dx::mbar_wait(dx::smem_u32(&bar), 0u, &abort_flag);
    *result = ok ? 1 : 2;
  }
}

}  // namespace

extern "C" {

int dx_fused_linear_ex(const void* X, const void* W, const void* bias, const void* R, void* Y,
                       int64_t M, int64_t N, int64_t K, int64_t ldx, int64_t ldw, int64_t ldr,
                       int64_t ldy, int dtype, int act, int kernel, void* workspace,
                       size_t workspace_bytes, void* stream) {
  Problem p{X, W, bias, R, Y, M, N, K, ldx, ldw, ldr, ldy, dtype, act, workspace, workspace_bytes,
            static_cast<cudaStream_t>(stream)};
  return run(p, kernel);
}

int dx_fused_linear(const void* X, const void* W, const void* bias, const void* R, void* Y,
                    int64_t M, int64_t N, int64_t K, int64_t ldx, int64_t ldw, int64_t ldr,
                    int64_t ldy, int dtype, int act, void* workspace, size_t workspace_bytes,
                    void* stream) {
  return dx_fused_linear_ex(X, W, bias, R, Y, M, N, K, ldx, ldw, ldr, ldy, dtype, act,
                            DX_KERNEL_AUTO, workspace, workspace_bytes, stream);
}

int dx_fused_linear_rowjob(const void* X, const void* W, const void* bias, const void* R, void* Y,
                           int64_t M, int64_t N, int64_t K, int64_t ldx, int64_t ldw,
                           int64_t ldr, int64_t ldy, int dtype, int act, int kernel,
                           void* workspace, size_t workspace_bytes, const dx_row_reduce_job* job,
                           void* stream) {
  t_last_error.clear();
  Problem p{X, W, bias, R, Y, M, N, K, ldx, ldw, ldr, ldy, dtype, act, workspace, workspace_bytes,
            static_cast<cudaStream_t>(stream)};
  dx::RowReduceArgs a{};
  if (job != nullptr) {
    const int rc = row_job_args(job, &a);
    if (rc) return rc;
    p.comm = &a;
    p.comm_dtype = job->dtype;
  }
  return run(p, kernel);
}

size_t dx_fused_linear_workspace_size(int64_t M, int64_t N, int64_t K, int dtype, int kernel) {
  t_last_error.clear();
  if (M <= 0 || N <= 0 || K <= 0 || dtype == DX_DTYPE_F32 || kernel == DX_KERNEL_SIMT) return 0;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || device_sms(dev, &sms) != DX_OK) return 0;
  if (kernel == DX_KERNEL_AUTO) kernel = dx_select_kernel(M, N, K, dtype);
  if (kernel == DX_KERNEL_DECODE) {
    if (M > kDecodeMaxM || (N + kDecodeTileN - 1) / kDecodeTileN > kDecodeMaxTiles) return 0;
    return decode_plan(M, N, K, sms).bytes;
  }
  if (kernel == DX_KERNEL_UMMA || kernel == DX_KERNEL_UMMA_1CTA) {
    const bool single = kernel == DX_KERNEL_UMMA_1CTA;
    const int slots = (M >= 256 && !single) ? pair_slots<256, __nv_bfloat16>(dev, sms) : 0;
    return plan_umma(M, N, K, sms, slots, true, single).bytes;
  }
  return 0;
}

int dx_fused_gated_linear(const void* X, const void* Wg, const void* Wu, const void* bias_g,
                          const void* bias_u, void* Y, int64_t M, int64_t N, int64_t K,
                          int64_t ldx, int64_t ldwg, int64_t ldwu, int64_t ldy, int dtype, int act,
                          int kernel, void* workspace, size_t workspace_bytes, void* stream) {
  Problem p{X, Wg, bias_g, nullptr, Y, M, N, K, ldx, ldwg, 0, ldy, dtype, act, workspace,
            workspace_bytes, static_cast<cudaStream_t>(stream)};
  p.gated = true;
  p.W2 = Wu;
  p.bias2 = bias_u;
  p.ldw2 = ldwu;
  return run(p, kernel);
}

int dx_fused_gated_linear_rowjob(const void* X, const void* Wg, const void* Wu,
                                 const void* bias_g, const void* bias_u, void* Y, int64_t M,
                                 int64_t N, int64_t K, int64_t ldx, int64_t ldwg, int64_t ldwu,
                                 int64_t ldy, int dtype, int act, int kernel, void* workspace,
                                 size_t workspace_bytes, const dx_row_reduce_job* job,
                                 void* stream) {
  t_last_error.clear();
  Problem p{X, Wg, bias_g, nullptr, Y, M, N, K, ldx, ldwg, 0, ldy, dtype, act, workspace,
            workspace_bytes, static_cast<cudaStream_t>(stream)};
  p.gated = true;
  p.W2 = Wu;
  p.bias2 = bias_u;
  p.ldw2 = ldwu;
  dx::RowReduceArgs a{};
  if (job != nullptr) {
    const int rc = row_job_args(job, &a);
    if (rc) return rc;
    p.comm = &a;
    p.comm_dtype = job->dtype;
  }
  return run(p, kernel);
}

size_t dx_fused_gated_linear_workspace_size(int64_t M, int64_t N, int64_t K, int dtype,
                                            int kernel) {
  t_last_error.clear();
  if (M <= 0 || N <= 0 || K <= 0 || dtype == DX_DTYPE_F32 || kernel == DX_KERNEL_SIMT) return 0;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || device_sms(dev, &sms) != DX_OK) return 0;
  const int tn = decode_min_tile_n(true);
  const bool fits = M <= kDecodeMaxM && (N + tn - 1) / tn <= kDecodeMaxTiles;
  if (kernel == DX_KERNEL_AUTO)
    kernel = (fits && decode_preferred(M, N, K, sms, true)) ? DX_KERNEL_DECODE : DX_KERNEL_UMMA;
  if (kernel == DX_KERNEL_DECODE && fits) return decode_plan(M, N, K, sms, true).bytes;
  return 0;  // the gated tensor-core kernels take no split tail
}

int dx_copy_2d_async(void* dst, size_t dst_pitch, const void* src, size_t src_pitch,
                     size_t width_bytes, size_t rows, void* stream) {
  t_last_error.clear();
  if (rows == 0 || width_bytes == 0) return DX_OK;
  if (dst == nullptr || src == nullptr || dst_pitch < width_bytes || src_pitch < width_bytes)
    return fail(DX_ERR_INVALID_ARGUMENT, "copy_2d: NULL pointer or pitch below the row width");
  const cudaError_t e = cudaMemcpy2DAsync(dst, dst_pitch, src, src_pitch, width_bytes, rows,
                                          cudaMemcpyDefault, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpy2DAsync");
  return DX_OK;
}

int dx_select_kernel(int64_t M, int64_t N, int64_t K, int dtype) {
  if (dtype == DX_DTYPE_F32 || K <= 0) return DX_KERNEL_SIMT;
  if ((K * 2) % 16 != 0 || (N * 2) % 16 != 0) return DX_KERNEL_SIMT;
  int sms = 148;  // B200; the device's own count when one is current
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || device_sms(dev, &sms) != DX_OK) {
    sms = 148;
    (void)cudaGetLastError();
    t_last_error.clear();  // no device: not an error of this query
  }
  if (M <= kDecodeMaxM && (N + kDecodeTileN - 1) / kDecodeTileN <= kDecodeMaxTiles &&
      decode_preferred(M, N, K, sms, false))
    return DX_KERNEL_DECODE;
  return DX_KERNEL_UMMA;
}

int dx_reduce_broadcast(void* const* P, int world, int rank, int64_t rows_per_rank, int64_t N,
                        int64_t ldp, const void* bias, const void* R, int64_t ldr,
                        void* const* Y, int64_t ldy, int dtype, void* stream) {
  t_last_error.clear();
  if (P == nullptr || Y == nullptr || world < 1 || world > 8 || rank < 0 || rank >= world)
    return fail(DX_ERR_INVALID_ARGUMENT, "reduce_broadcast: bad P/Y/world/rank");
  if (dtype != DX_DTYPE_F16 && dtype != DX_DTYPE_BF16)
    return fail(DX_ERR_UNSUPPORTED, "reduce_broadcast supports fp16/bf16");
  if (rows_per_rank <= 0 || N <= 0 || N % 8 != 0 || ldp < N || ldy < N || ldp % 8 != 0 ||
      ldy % 8 != 0 || (R != nullptr && (ldr < N || ldr % 8 != 0)))
    return fail(DX_ERR_INVALID_ARGUMENT, "reduce_broadcast needs N %% 8 == 0 and pitches >= N, "
                "multiples of 8");
  if ((bias != nullptr && !aligned16(bias)) || (R != nullptr && !aligned16(R)))
    return fail(DX_ERR_INVALID_ARGUMENT, "reduce_broadcast needs 16-byte-aligned buffers");
  dx::RankPtrs pp{}, yp{};
  for (int r = 0; r < world; ++r) {
    if (P[r] == nullptr || !aligned16(P[r]) || Y[r] == nullptr || !aligned16(Y[r]))
      return fail(DX_ERR_INVALID_ARGUMENT, "buffer of rank %d is NULL or not 16-byte aligned", r);
    pp.p[r] = P[r];
    yp.p[r] = Y[r];
  }
  int dev = 0, sms = 0, rc;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if ((rc = device_sms(dev, &sms))) return rc;
  if ((rc = install_status_mirror(dev, static_cast<cudaStream_t>(stream)))) return rc;
  if ((rc = check_status_mirror(dev))) return rc;
  const long long work = rows_per_rank * (N / 8);
  const int grid = static_cast<int>(std::max<long long>(
      1, std::min<long long>((work + 511) / 512, 8LL * sms)));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  set_plan("reduce_broadcast world=%d rows=%lld N=%lld grid=%d", world, (long long)rows_per_rank,
           (long long)N, grid);
  if (dtype == DX_DTYPE_F16)
    dx::reduce_broadcast_kernel<__half><<<grid, 256, 0, s>>>(
        pp, world, rank, static_cast<int>(rows_per_rank), static_cast<int>(N), ldp,
        static_cast<const __half*>(bias), static_cast<const __half*>(R), ldr, yp, ldy);
  else
    dx::reduce_broadcast_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
        pp, world, rank, static_cast<int>(rows_per_rank), static_cast<int>(N), ldp,
        static_cast<const __nv_bfloat16*>(bias), static_cast<const __nv_bfloat16*>(R), ldr, yp,
        ldy);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch reduce_broadcast_kernel");
  return DX_OK;
}

int dx_row_flag_words(void) { return dx::kRowFlagWords; }

int dx_row_reduce(const dx_row_reduce_job* job, int grid, void* stream) {
  t_last_error.clear();
  dx::RowReduceArgs a{};
  int rc = row_job_args(job, &a);
  if (rc) return rc;
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if ((rc = stream_sms(s, dev, &sms))) return rc;
  if ((rc = install_status_mirror(dev, s))) return rc;
  if ((rc = check_status_mirror(dev))) return rc;
  return launch_row_reduce(a, job->dtype, sms, grid, s);
}

// ------------------------------------------------------------- plans
// A plan fixes everything the reference's compile step fixes (shape, dtype,
// op sequence; doc/kvlang-to-tilelang-interface.md:60-77) so that a call
// needs only the docs' runtime arguments: pointers and a stream.
struct dx_plan {
  int64_t M, N, K;
  int dtype, act, kernel;
  float alpha;
  void* ws;
  size_t ws_bytes;
};

int dx_plan_create(dx_plan** out, int64_t M, int64_t N, int64_t K, int dtype, int act, float alpha,
                   int kernel) {
  t_last_error.clear();
  if (out == nullptr) return fail(DX_ERR_INVALID_ARGUMENT, "plan output pointer is NULL");
  *out = nullptr;
  Problem probe{nullptr, nullptr, nullptr, nullptr, nullptr, M, N, K, std::max<int64_t>(K, 1), N,
                0, N, dtype, act, nullptr, 0, nullptr};
  // Shape/enum checks only (pointers are supplied per call).
  if (M < 0 || N < 0 || K < 0)
    return fail(DX_ERR_INVALID_ARGUMENT, "negative shape M=%lld N=%lld K=%lld", (long long)M,
                (long long)N, (long long)K);
  probe.M = 0;  // skip the pointer checks of validate()
  int rc = validate(probe, kernel);
  if (rc) return rc;
  if (M > 0x7fffffffLL || N > 0x7fffffffLL || K > 0x7fffffffLL)
    return fail(DX_ERR_UNSUPPORTED, "dimension above 2^31-1");
  dx_plan* pl = new (std::nothrow) dx_plan{M, N, K, dtype, act, kernel, alpha, nullptr, 0};
  if (pl == nullptr) return fail(DX_ERR_UNSUPPORTED, "out of host memory");
  *out = pl;
  return DX_OK;
}

size_t dx_plan_workspace_size(const dx_plan* plan) {
  if (plan == nullptr) return 0;
  return dx_fused_linear_workspace_size(plan->M, plan->N, plan->K, plan->dtype, plan->kernel);
}

int dx_plan_set_workspace(dx_plan* plan, void* workspace, size_t bytes) {
  t_last_error.clear();
  if (plan == nullptr) return fail(DX_ERR_INVALID_ARGUMENT, "plan is NULL");
  plan->ws = workspace;
  plan->ws_bytes = workspace != nullptr ? bytes : 0;
  return DX_OK;
}

int dx_plan_call_residual(const dx_plan* plan, const void* x, const void* W, const void* b,
                          const void* r, void* out, void* stream) {
  t_last_error.clear();
  if (plan == nullptr) return fail(DX_ERR_INVALID_ARGUMENT, "plan is NULL");
  Problem p{x,          W,           b, r,        out, plan->M, plan->N, plan->K,
            std::max<int64_t>(plan->K, 1), plan->N, plan->N, plan->N, plan->dtype, plan->act,
            plan->ws,   plan->ws_bytes, static_cast<cudaStream_t>(stream)};
  p.alpha = plan->alpha;
  return run(p, plan->kernel);
}

int dx_plan_call(const dx_plan* plan, const void* x, const void* W, const void* b, void* out,
                 void* stream) {
  return dx_plan_call_residual(plan, x, W, b, nullptr, out, stream);
}

int dx_plan_destroy(dx_plan* plan) {
  delete plan;
  return DX_OK;
}

const char* dx_last_error_string(void) { return t_last_error.c_str(); }

const char* dx_last_launch_plan(void) { return t_last_plan.c_str(); }

int dx_set_trace_buffer(void* device_buffer, size_t bytes) {
  t_last_error.clear();
  if (device_buffer != nullptr && (reinterpret_cast<uintptr_t>(device_buffer) & 7u) != 0)
    return fail(DX_ERR_INVALID_ARGUMENT, "trace buffer must be 8-byte aligned");
  g_trace_bytes.store(device_buffer != nullptr ? bytes : 0);
  g_trace.store(static_cast<unsigned long long*>(device_buffer));
  return DX_OK;
}

int dx_device_status(void* stream, int* status) {
  t_last_error.clear();
  if (status == nullptr) return fail(DX_ERR_INVALID_ARGUMENT, "status is NULL");
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  int v = 0;
  e = cudaMemcpyFromSymbol(&v, dx::g_device_status, sizeof(int));
  if (e != cudaSuccess) return cuda_fail(e, "read device status");
  if (v != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(dx::g_device_status, &zero, sizeof(int));
    if (e != cudaSuccess) return cuda_fail(e, "clear device status");
  }
  int dev = 0;
  if (g_host_status != nullptr && cudaGetDevice(&dev) == cudaSuccess && dev >= 0 &&
      dev < kMaxDevices) {
    volatile int* mirror = reinterpret_cast<volatile int*>(g_host_status) + dev;
    v |= *mirror;
    *mirror = 0;
  }
  *status = v;
  return DX_OK;
}

int dx_selftest_bounded_wait(int* result, void* stream) {
  t_last_error.clear();
  if (result == nullptr) return fail(DX_ERR_INVALID_ARGUMENT, "result is NULL");
  selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(result);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch selftest_wait_kernel");
  return DX_OK;
}

int dx_kernel_arch(int* binary_version, int* ptx_version) {
  t_last_error.clear();
  if (binary_version == nullptr || ptx_version == nullptr)
    return fail(DX_ERR_INVALID_ARGUMENT, "dx_kernel_arch: NULL output");
  cudaFuncAttributes fa{};
  const cudaError_t e = cudaFuncGetAttributes(
      &fa, reinterpret_cast<const void*>(dx::umma2_fused_linear_kernel<256, __nv_bfloat16>));
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncGetAttributes");
  *binary_version = fa.binaryVersion;
  *ptx_version = fa.ptxVersion;
  return DX_OK;
}

int dx_version(void) { return 100; }

}  // extern "C"

// =========================================================================
// Decode entry point that allocates nothing.
//
// The decode kernel needs split-K scratch (per-tile tickets and fp32 partial
// sums).  dx_fused_linear takes it from the caller as a workspace; some
// callers have none to give and may not allocate: a runtime that owns every
// device buffer through its own heap manager and hands a kernel only raw
// pointers and a stream (the `kernel_fn(x, W, b, out, stream)` shape of the
// kvlang dispatcher) cannot call cudaMalloc behind its allocator's back.  For
// them the scratch lives in one fixed device array inside this library,
// kStaticScratchBytes large; every GPU that loads the library holds it until
// the process exits.
//
// Set-up: the first split-K call in a context (normally once per device)
// resolves the array's device address with cudaGetSymbolAddress while that
// device is current, and caches it by context.  Make that first call before
// any stream capture.
// All calls on a device share the array and it keeps the last call's
// contents; a split-K call clears the tickets on the caller's stream (the
// partial sums are written before they are read); a call whose plan streams
// whole tiles uses no scratch and clears nothing.
// Calls that overlap on the GPU (different streams, or concurrent host
// threads) race on the shared scratch — serialise them.
// =========================================================================
namespace {

constexpr size_t kStaticScratchBytes = size_t(8) << 20;  // 8 MiB per device
static __device__ __align__(256) unsigned char g_static_decode_scratch[kStaticScratchBytes];

std::mutex g_static_scratch_mu;
std::map<unsigned long long, void*> g_static_scratch_addr;  // by context id

// Device address of the static scratch in the current context.  Each context
// holds its own copy of the array (the module is loaded per context), so the
// address is cached per context id, not per device ordinal.
int static_scratch_address(void** out) {
  std::lock_guard<std::mutex> lk(g_static_scratch_mu);
  const unsigned long long ctx = current_context_id();
  auto it = ctx != 0 ? g_static_scratch_addr.find(ctx) : g_static_scratch_addr.end();
  if (it != g_static_scratch_addr.end()) {
    *out = it->second;
    return DX_OK;
  }
  void* ptr = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&ptr, g_static_decode_scratch);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(static decode scratch)");
  if (ptr == nullptr) return fail(DX_ERR_CUDA, "static decode scratch has no device address");
  const unsigned long long now = current_context_id();  // current after the runtime call
  if (now != 0) g_static_scratch_addr[now] = ptr;
  *out = ptr;
  return DX_OK;
}

}  // namespace

extern "C" int dx_fused_linear_decode_noalloc(const void* X, const void* W, const void* bias,
                                              const void* R, void* Y, int64_t M, int64_t N,
                                              int64_t K, int64_t ldx, int64_t ldw, int64_t ldr,
                                              int64_t ldy, int dtype, int act, void* stream) {
  t_last_error.clear();
  Problem p{X,   W,   bias, R,     Y,   M,       N, K, ldx, ldw, ldr, ldy,
            dtype, act, nullptr, 0, static_cast<cudaStream_t>(stream)};
  int rc = validate(p, DX_KERNEL_DECODE);
  if (rc) return rc;
  if (M == 0 || N == 0) return DX_OK;
  if (!decode_eligible(p))
    return fail(DX_ERR_UNSUPPORTED,
                "dx_fused_linear_decode_noalloc needs fp16/bf16, 0 < K, M <= %d, and "
                "16-byte-aligned X/W with row pitches that are multiples of 16 bytes",
                kDecodeMaxM);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  int sms = 0;
  if ((rc = device_sms(dev, &sms))) return rc;
  if ((rc = check_status_mirror(dev))) return rc;
  const DecodePlan d = decode_plan(M, N, K, sms);
  if (d.bytes > kStaticScratchBytes)
    return fail(DX_ERR_WORKSPACE,
                "dx_fused_linear_decode_noalloc: this problem needs %zu bytes of split-K scratch "
                "but the library's static scratch holds %zu; use dx_fused_linear with a workspace",
                d.bytes, kStaticScratchBytes);
  if (!load_encode_fn())
    return fail(DX_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if (d.bytes > 0) {
    // Split-K plan: its tickets must start at zero (an aborted earlier call
    // may have left some set); the partial sums are always written before
    // they are read.  A whole-tile plan touches no scratch at all.
    void* scratch = nullptr;
    if ((rc = static_scratch_address(&scratch))) return rc;
    e = cudaMemsetAsync(scratch, 0, d.ticket_bytes, p.stream);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(static decode scratch tickets)");
    p.ws = scratch;
    p.ws_bytes = kStaticScratchBytes;
  }
  if (dtype == DX_DTYPE_F16) {
    if (d.mn == 16) return launch_decode<16, __half>(p, dev, sms, d);
    if (d.mn == 32) return launch_decode<32, __half>(p, dev, sms, d);
    return launch_decode<64, __half>(p, dev, sms, d);
  }
  if (d.mn == 16) return launch_decode<16, __nv_bfloat16>(p, dev, sms, d);
  if (d.mn == 32) return launch_decode<32, __nv_bfloat16>(p, dev, sms, d);
  return launch_decode<64, __nv_bfloat16>(p, dev, sms, d);
}
