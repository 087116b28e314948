// A non-Python caller of the engine, as the reference design docs' C++
// runtime would be (doc/kernel-compiler-analysis.md:113-134,
// doc/kvlang-to-tilelang-interface.md:79-98): dlopen the library, compile a
// plan once per (pattern, shape, dtype), then call it with raw device
// pointers and a stream — the docs' kernel_fn(x_ptr, W_ptr, b_ptr, out_ptr,
// cuda_stream).  The program owns every device buffer.
//
//   dx_runtime_demo <path to libdeepx_fused.so>
//
// Checks against a double-precision host reference:
//   linear_relu, fp16, x[512,256] W[256,512] b[512]   (the docs' example shape)
//   linear_gelu (tanh), fp16, x[16,1024] W[1024,2048] (skinny M: needs a workspace)
//   mlp_residual, fp16, x[256,256] W1[256,1024] W2[1024,256]: the two-plan chain
//     y = gelu(x W1 + b1) W2 + b2 + x (dx_plan_call, then dx_plan_call_residual)
// and prints one line per case; exit status 0 when all are within the fp16
// tolerance (|diff| <= 2e-2 + 2e-2 |ref|).
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <dlfcn.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <vector>

#include "deepx_fused.h"

namespace {

struct Api {
  int (*plan_create)(dx_plan**, int64_t, int64_t, int64_t, int, int, float, int);
  size_t (*plan_workspace_size)(const dx_plan*);
  int (*plan_set_workspace)(dx_plan*, void*, size_t);
  int (*plan_call)(const dx_plan*, const void*, const void*, const void*, void*, void*);
  int (*plan_call_residual)(const dx_plan*, const void*, const void*, const void*, const void*,
                            void*, void*);
  int (*plan_destroy)(dx_plan*);
  const char* (*last_error)(void);
  int (*version)(void);
};

template <typename F>
bool resolve(void* h, const char* name, F* out) {
  *out = reinterpret_cast<F>(dlsym(h, name));
  if (*out == nullptr) std::fprintf(stderr, "missing symbol %s\n", name);
  return *out != nullptr;
}

uint32_t g_state = 12345u;
float uniform() {  // deterministic LCG in [-1, 1)
  g_state = g_state * 1664525u + 1013904223u;
  return static_cast<float>(g_state >> 8) / 8388608.0f - 1.0f;
}

double act(double v, int a) {
  if (a == DX_ACT_RELU) return v > 0.0 ? v : 0.0;
  if (a == DX_ACT_GELU_TANH)
    return 0.5 * v * (1.0 + std::tanh(0.7978845608028654 * (v + 0.044715 * v * v * v)));
  return v;
}

#define CK(x)                                                                       \
  do {                                                                              \
    cudaError_t e_ = (x);                                                           \
    if (e_ != cudaSuccess) {                                                        \
      std::fprintf(stderr, "%s: %s\n", #x, cudaGetErrorString(e_));                \
      return false;                                                                 \
    }                                                                               \
  } while (0)

bool run_plan(const Api& api, const char* name, int64_t M, int64_t N, int64_t K, int a,
              cudaStream_t stream) {
  std::vector<__half> x(M * K), w(K * N), b(N), y(M * N);
  std::vector<double> xd(M * K), wd(K * N), bd(N);
  const float ws = 1.0f / std::sqrt(static_cast<float>(K));
  for (size_t i = 0; i < x.size(); ++i) { x[i] = __float2half(uniform()); xd[i] = __half2float(x[i]); }
  for (size_t i = 0; i < w.size(); ++i) { w[i] = __float2half(uniform() * ws); wd[i] = __half2float(w[i]); }
  for (size_t i = 0; i < b.size(); ++i) { b[i] = __float2half(0.1f * uniform()); bd[i] = __half2float(b[i]); }

  void *dx = nullptr, *dw = nullptr, *db = nullptr, *dy = nullptr, *dws = nullptr;
  CK(cudaMalloc(&dx, x.size() * 2));
  CK(cudaMalloc(&dw, w.size() * 2));
  CK(cudaMalloc(&db, b.size() * 2));
  CK(cudaMalloc(&dy, y.size() * 2));
  CK(cudaMemcpy(dx, x.data(), x.size() * 2, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(dw, w.data(), w.size() * 2, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(db, b.data(), b.size() * 2, cudaMemcpyHostToDevice));

  dx_plan* plan = nullptr;  // compile step: shape, dtype and op sequence fixed
  if (api.plan_create(&plan, M, N, K, DX_DTYPE_F16, a, 1.0f, DX_KERNEL_AUTO) != DX_OK) {
    std::fprintf(stderr, "dx_plan_create: %s\n", api.last_error());
    return false;
  }
  const size_t need = api.plan_workspace_size(plan);
  if (need > 0) {  // caller-owned, zero-filled once before first use
    CK(cudaMalloc(&dws, need));
    CK(cudaMemset(dws, 0, need));
    api.plan_set_workspace(plan, dws, need);
  }
  bool ok = true;
  for (int call = 0; call < 2 && ok; ++call) {  // a plan is called many times
    if (api.plan_call(plan, dx, dw, db, dy, stream) != DX_OK) {
      std::fprintf(stderr, "dx_plan_call: %s\n", api.last_error());
      ok = false;
    }
  }
  CK(cudaStreamSynchronize(stream));
  CK(cudaMemcpy(y.data(), dy, y.size() * 2, cudaMemcpyDeviceToHost));
  double max_err = 0.0;
  int bad = 0;
  for (int64_t m = 0; m < M && ok; ++m)
    for (int64_t n = 0; n < N; ++n) {
      double s = bd[n];
      for (int64_t k = 0; k < K; ++k) s += xd[m * K + k] * wd[k * N + n];
      const double ref = act(s, a), got = __half2float(y[m * N + n]);
      const double err = std::fabs(got - ref);
      max_err = err > max_err ? err : max_err;
      if (err > 2e-2 + 2e-2 * std::fabs(ref)) ++bad;
    }
  std::printf("%s M=%lld N=%lld K=%lld workspace=%zu max_abs_err=%.3g bad=%d\n", name,
              static_cast<long long>(M), static_cast<long long>(N), static_cast<long long>(K),
              need, max_err, bad);
  api.plan_destroy(plan);
  cudaFree(dx);
  cudaFree(dw);
  cudaFree(db);
  cudaFree(dy);
  if (dws != nullptr) cudaFree(dws);
  return ok && bad == 0;
}

// The MLP chain as a dispatcher composes it from two compiled plans; the
// hidden activations stay on the device between the calls.
bool run_mlp_chain(const Api& api, int64_t M, int64_t K, int64_t H, cudaStream_t stream) {
  std::vector<__half> x(M * K), w1(K * H), b1(H), w2(H * K), b2(K), y(M * K);
  std::vector<double> xd(M * K), w1d(K * H), b1d(H), w2d(H * K), b2d(K);
  auto fill = [](std::vector<__half>& v, std::vector<double>& d, float scale) {
    for (size_t i = 0; i < v.size(); ++i) {
      v[i] = __float2half(uniform() * scale);
      d[i] = __half2float(v[i]);
    }
  };
  fill(x, xd, 1.0f);
  fill(w1, w1d, 1.0f / std::sqrt(static_cast<float>(K)));
  fill(b1, b1d, 0.1f);
  fill(w2, w2d, 1.0f / std::sqrt(static_cast<float>(H)));
  fill(b2, b2d, 0.1f);
  void *dx = nullptr, *dw1 = nullptr, *db1 = nullptr, *dw2 = nullptr, *db2 = nullptr,
       *dh = nullptr, *dy = nullptr;
  CK(cudaMalloc(&dx, x.size() * 2));
  CK(cudaMalloc(&dw1, w1.size() * 2));
  CK(cudaMalloc(&db1, b1.size() * 2));
  CK(cudaMalloc(&dw2, w2.size() * 2));
  CK(cudaMalloc(&db2, b2.size() * 2));
  CK(cudaMalloc(&dh, M * H * 2));
  CK(cudaMalloc(&dy, y.size() * 2));
  CK(cudaMemcpy(dx, x.data(), x.size() * 2, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(dw1, w1.data(), w1.size() * 2, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(db1, b1.data(), b1.size() * 2, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(dw2, w2.data(), w2.size() * 2, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(db2, b2.data(), b2.size() * 2, cudaMemcpyHostToDevice));
  dx_plan *up = nullptr, *down = nullptr;
  if (api.plan_create(&up, M, H, K, DX_DTYPE_F16, DX_ACT_GELU_TANH, 1.0f, DX_KERNEL_AUTO) != DX_OK ||
      api.plan_create(&down, M, K, H, DX_DTYPE_F16, DX_ACT_NONE, 1.0f, DX_KERNEL_AUTO) != DX_OK) {
    std::fprintf(stderr, "dx_plan_create: %s\n", api.last_error());
    return false;
  }
  void* dws[2] = {nullptr, nullptr};
  dx_plan* plans[2] = {up, down};
  for (int i = 0; i < 2; ++i) {  // one caller-owned, zero-filled workspace per plan
    const size_t need = api.plan_workspace_size(plans[i]);
    if (need > 0) {
      CK(cudaMalloc(&dws[i], need));
      CK(cudaMemset(dws[i], 0, need));
      api.plan_set_workspace(plans[i], dws[i], need);
    }
  }
  bool ok = true;
  for (int call = 0; call < 2 && ok; ++call) {
    if (api.plan_call(up, dx, dw1, db1, dh, stream) != DX_OK ||
        api.plan_call_residual(down, dh, dw2, db2, dx, dy, stream) != DX_OK) {
      std::fprintf(stderr, "plan call: %s\n", api.last_error());
      ok = false;
    }
  }
  CK(cudaStreamSynchronize(stream));
  CK(cudaMemcpy(y.data(), dy, y.size() * 2, cudaMemcpyDeviceToHost));
  double max_err = 0.0;
  int bad = 0;
  std::vector<double> h(H);
  for (int64_t m = 0; m < M && ok; ++m) {
    for (int64_t j = 0; j < H; ++j) {
      double s = b1d[j];
      for (int64_t k = 0; k < K; ++k) s += xd[m * K + k] * w1d[k * H + j];
      h[j] = act(s, DX_ACT_GELU_TANH);
    }
    for (int64_t n = 0; n < K; ++n) {
      double s = b2d[n] + xd[m * K + n];
      for (int64_t j = 0; j < H; ++j) s += h[j] * w2d[j * K + n];
      const double err = std::fabs(__half2float(y[m * K + n]) - s);
      max_err = err > max_err ? err : max_err;
      if (err > 2e-2 + 2e-2 * std::fabs(s)) ++bad;
    }
  }
  std::printf("mlp_residual M=%lld K=%lld H=%lld plans=2 max_abs_err=%.3g bad=%d\n",
              static_cast<long long>(M), static_cast<long long>(K), static_cast<long long>(H),
              max_err, bad);
  api.plan_destroy(up);
  api.plan_destroy(down);
  for (void* p : {dx, dw1, db1, dw2, db2, dh, dy, dws[0], dws[1]})
    if (p != nullptr) cudaFree(p);
  return ok && bad == 0;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc < 2) {
    std::fprintf(stderr, "usage: %s <libdeepx_fused.so>\n", argv[0]);
    return 2;
  }
  void* h = dlopen(argv[1], RTLD_NOW | RTLD_LOCAL);
  if (h == nullptr) {
    std::fprintf(stderr, "dlopen: %s\n", dlerror());
    return 2;
  }
  Api api{};
  if (!(resolve(h, "dx_plan_create", &api.plan_create) &&
        resolve(h, "dx_plan_workspace_size", &api.plan_workspace_size) &&
        resolve(h, "dx_plan_set_workspace", &api.plan_set_workspace) &&
        resolve(h, "dx_plan_call", &api.plan_call) &&
        resolve(h, "dx_plan_call_residual", &api.plan_call_residual) &&
        resolve(h, "dx_plan_destroy", &api.plan_destroy) &&
        resolve(h, "dx_last_error_string", &api.last_error) &&
        resolve(h, "dx_version", &api.version)))
    return 2;
  std::printf("engine ABI version %d\n", api.version());
  cudaStream_t stream;
  if (cudaStreamCreate(&stream) != cudaSuccess) return 2;
  const bool ok = run_plan(api, "linear_relu", 512, 512, 256, DX_ACT_RELU, stream) &&
                  run_plan(api, "linear_gelu", 16, 2048, 1024, DX_ACT_GELU_TANH, stream) &&
                  run_mlp_chain(api, 256, 256, 1024, stream);
  cudaStreamDestroy(stream);
  return ok ? 0 : 1;
}
