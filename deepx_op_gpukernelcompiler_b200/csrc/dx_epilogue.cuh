// dx_epilogue.cuh — element types and the fused epilogue math shared by all
// kernels: y = act(acc + bias) (+ residual), computed in fp32.
//
// Activation definitions follow the reference:
//   relu            torch.relu                     (fusion.py:88)
//   gelu (tanh)     F.gelu(approximate='tanh')     (fusion.py:89)
//   gelu (erf)      0.5*x*(erf(x/sqrt(2)) + 1)     (kernel_triton.py:61,
//                                                   kernel_tilelang.py:17)
//   silu / swish    x * sigmoid(x)                 (fusion.py:90-91,
//                                                   kernel_triton.py:63)
// The exact forms call CUDA's tanhf / erff / expf and IEEE division (used
// for fp32 outputs).  For fp16/bf16 outputs (kFast) GELU-tanh uses the
// hardware tanh (tanh.approx.f32, max relative error about 2^-11) and SiLU
// the identity sigmoid(x) = (1 + tanh(x/2)) / 2 on the same instruction: one
// special-function op per element instead of an exponential and a division.
// Its absolute error is at most about 3e-4 * |x| where tanh(x/2) is not yet
// +-1 in fp32 (|x| < 18), i.e. below 6e-3, and nothing can overflow;
// GELU-erf takes erfc from a published rational approximation (gelu_erf_hw,
// absolute error below 5e-7).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

namespace dx {

enum Act : int { kActNone = 0, kActRelu = 1, kActGeluTanh = 2, kActGeluErf = 3, kActSilu = 4 };

__device__ __forceinline__ float tanh_hw(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float ex2_hw(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float rcp_hw(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// GELU in its erf form, 0.5 x (1 + erf(x / sqrt 2)), for fp16/bf16 outputs.
// 1 + erf(-a) = erfc(a) comes straight from Abramowitz & Stegun, Handbook of
// Mathematical Functions, formula 7.1.26 (Hastings' rational approximation,
// |error| <= 1.5e-7):
//   erfc(a) = t (a1 + t (a2 + t (a3 + t (a4 + t a5)))) exp(-a^2),
//   t = 1 / (1 + p a), a >= 0,
// so the negative tail has no 1 + erf cancellation.  In fp32 the GELU error
// is below 5e-7 absolute, and below 6e-5 relative for x >= -3: under half an
// fp16 ulp.  Two special-function ops (rcp, ex2) and ~12 FMA-pipe ops.
__device__ __forceinline__ float gelu_erf_hw(float x) {
  const float a = fabsf(x) * 0.7071067811865476f;
  const float t = rcp_hw(fmaf(0.3275911f, a, 1.0f));
  float q = fmaf(1.061405429f, t, -1.453152027f);
  q = fmaf(q, t, 1.421413741f);
  q = fmaf(q, t, -0.284496736f);
  q = fmaf(q, t, 0.254829592f);
  const float ec = q * t * ex2_hw(-1.4426950408889634f * a * a);  // erfc(a)
  const float h = 0.5f * x;
  return x >= 0.0f ? fmaf(-h, ec, x) : h * ec;  // x - h erfc(a) | h erfc(a)
}

template <bool kFast = true>
__device__ __forceinline__ float act_apply(float x, int act) {
  switch (act) {
    case kActRelu:
      return fmaxf(x, 0.0f);
    case kActGeluTanh: {
      // sqrt(2/pi) * (x + 0.044715 x^3)
      const float u = 0.7978845608028654f * fmaf(0.044715f * x, x * x, x);
      return 0.5f * x * (1.0f + (kFast ? tanh_hw(u) : tanhf(u)));
    }
    case kActGeluErf:
      return kFast ? gelu_erf_hw(x) : 0.5f * x * (1.0f + erff(x * 0.7071067811865476f));
    case kActSilu:
      if (kFast) {
        const float h = 0.5f * x;
        return fmaf(h, tanh_hw(h), h);  // x * (1 + tanh(x/2)) / 2
      }
      return x / (1.0f + expf(-x));
    default:
      return x;
  }
}

template <int A, bool kFast, int N>
__device__ __forceinline__ void act_loop(float (&v)[N]) {
#pragma unroll
  for (int j = 0; j < N; ++j) v[j] = act_apply<kFast>(v[j], A);
}

// The activation over a register array, the switch outside the element
// loop: each case is straight-line code whose independent per-element
// chains (erfc polynomial, tanh) the compiler interleaves, instead of one
// branch per element.
template <bool kFast = true, int N>
__device__ __forceinline__ void act_apply_all(float (&v)[N], int act) {
  switch (act) {
    case kActRelu: act_loop<kActRelu, kFast>(v); break;
    case kActGeluTanh: act_loop<kActGeluTanh, kFast>(v); break;
    case kActGeluErf: act_loop<kActGeluErf, kFast>(v); break;
    case kActSilu: act_loop<kActSilu, kFast>(v); break;
    default: break;
  }
}

template <typename T>
struct ElemTraits;

template <>
struct ElemTraits<float> {
  static constexpr bool kIsBf16 = false;
  __device__ __forceinline__ static float to_float(float v) { return v; }
  __device__ __forceinline__ static float from_float(float v) { return v; }
};

template <>
struct ElemTraits<__half> {
  static constexpr bool kIsBf16 = false;
  __device__ __forceinline__ static float to_float(__half v) { return __half2float(v); }
  __device__ __forceinline__ static __half from_float(float v) { return __float2half_rn(v); }
  // Two fp32 values -> packed pair (low half = first).
  __device__ __forceinline__ static uint32_t pack2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ __forceinline__ static float2 unpack2(uint32_t u) {
    __half2 h = *reinterpret_cast<__half2*>(&u);
    return __half22float2(h);
  }
};

template <>
struct ElemTraits<__nv_bfloat16> {
  static constexpr bool kIsBf16 = true;
  __device__ __forceinline__ static float to_float(__nv_bfloat16 v) { return __bfloat162float(v); }
  __device__ __forceinline__ static __nv_bfloat16 from_float(float v) {
    return __float2bfloat16_rn(v);
  }
  __device__ __forceinline__ static uint32_t pack2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ __forceinline__ static float2 unpack2(uint32_t u) {
    __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162*>(&u);
    return __bfloat1622float2(h);
  }
};

}  // namespace dx
